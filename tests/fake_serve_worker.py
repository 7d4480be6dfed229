"""Stand-in for the engine's serving worker (voxq_engine_run --serve), for host-side tests.

Speaks the same line protocol: prints {"ready": ...}, then answers each request line
"INDEX TOKENS TOKEN_SEED PATCHES" with one JSON line until "quit".  Its failure modes
are set by the environment (no GPU is involved):
  FAKE_SLEEP        seconds per patch (default 0.01)
  FAKE_HANG_AFTER   after this many answers, stop answering (sleeps until killed)
  FAKE_EXIT_AFTER   after this many answers, exit with status 3
  FAKE_NO_READY     never print the ready line (exit at once)
  FAKE_TAG          a string copied into every answer
"""
import json
import os
import sys
import time


def main():
    if os.environ.get("FAKE_NO_READY"):
        return 4
    sleep = float(os.environ.get("FAKE_SLEEP", "0.01"))
    hang = int(os.environ.get("FAKE_HANG_AFTER", "-1"))
    exit_after = int(os.environ.get("FAKE_EXIT_AFTER", "-1"))
    tag = os.environ.get("FAKE_TAG", "")
    print(json.dumps({"ready": True, "gpu": os.environ.get("CUDA_VISIBLE_DEVICES")}), flush=True)
    answered = 0
    for line in sys.stdin:
        if line.startswith("quit"):
            break
        if answered == hang:
            time.sleep(3600)
        if answered == exit_after:
            return 3
        idx, tokens, seed, patches = (int(x) for x in line.split())
        time.sleep(sleep * patches)
        print(json.dumps({"utt": idx, "tokens": tokens, "token_seed": seed, "patches": patches,
                          "latent_floats": 256 * patches, "audio_s": 0.16 * patches, "generate_s": sleep * patches,
                          "weight_bytes": 1000 * patches, "tag": tag, "pid": os.getpid()}), flush=True)
        answered += 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
