"""The engine's transformer block on the device (voxq_transformer_block_forward).

Oracle: a float64 numpy restatement of transformer_block_forward
(src/nn.c:579-700) and what it calls: RMSNorm (src/tensor.c:811-849),
attention_forward (src/nn.c:208-530) with RoPE (src/tensor.c:883-950), the
KV-cache write, the additive mask and softmax (src/tensor.c:710-752), and
swiglu_forward (src/nn.c:100-170).  The projection weights are exactly
representable in the tested format (every 32-weight block holds its format's
lowest and highest code on a power-of-two grid), so quantization at upload is
the identity and the oracle multiplies by the same weights.

Cases follow how the engine calls the block: a DiT-style call that fills a
fresh cache (pos 0, seq = cache length, no mask, no RoPE); a causal prefill
into a longer cache with RoPE; single-token decode steps that read the rows
earlier calls wrote (the device mirror); a host cache changed behind the
library's back (the mirror must notice and re-read it); a restart at pos 0 on
the same cache; batch rows both below (GEMV) and above (GEMM) 8.  Checked:
the block output and the cache rows written back to the host.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

import voxq

pytestmark = pytest.mark.gpu

TOL = 1e-3  # |out - ref| <= TOL * (|ref| + rms(ref))


def exact_weight(rng, n, k, qname):
    """[n, k] weights on the format's grid with every 32-block spanning its full code range."""
    if qname == "q8":
        q = rng.integers(0, 256, size=(n, k))
        q[:, 0::32], q[:, 1::32] = 0, 255
        return ((q - 128) * 2.0 ** -11).astype(np.float32)
    q = rng.integers(0, 16, size=(n, k))
    q[:, 0::32], q[:, 1::32] = 0, 15
    return ((q - 8) * 2.0 ** -7).astype(np.float32)


def rmsnorm(x, w, eps):
    d = x.shape[-1]
    ss = (np.where(np.isnan(x), 0.0, x).astype(np.float64) ** 2).sum(-1, keepdims=True)
    return x.astype(np.float64) / np.sqrt(ss / d + eps) * w


def rope(t, freqs, pos):
    """t [B, heads, S, hd]; freqs [positions, hd/2, 2] (cos, sin)."""
    half = t.shape[-1] // 2
    S = t.shape[2]
    c = freqs[pos:pos + S, :, 0][None, None]
    s = freqs[pos:pos + S, :, 1][None, None]
    x0, x1 = t[..., :half], t[..., half:]
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)


def block_ref(x, W, ck, cv, mask, freqs, pos, H, KVH, hd, eps):
    """Returns out and updates the float64 caches ck, cv [B, KVH, max_seq, hd] in place."""
    B, S, D = x.shape
    n = rmsnorm(x, W["n1"], eps)
    q = (n @ W["wq"].T).reshape(B, S, H, hd).transpose(0, 2, 1, 3)
    k = (n @ W["wk"].T).reshape(B, S, KVH, hd).transpose(0, 2, 1, 3)
    v = (n @ W["wv"].T).reshape(B, S, KVH, hd).transpose(0, 2, 1, 3)
    if freqs is not None:
        q, k = rope(q, freqs, pos), rope(k, freqs, pos)
    ck[:, :, pos:pos + S] = k
    cv[:, :, pos:pos + S] = v
    L = pos + S
    kk = np.repeat(ck[:, :, :L], H // KVH, axis=1)
    vv = np.repeat(cv[:, :, :L], H // KVH, axis=1)
    sc = q @ kk.transpose(0, 1, 3, 2) / np.sqrt(hd)
    if mask is not None:
        r, c = min(mask.shape[0], S), min(mask.shape[1], L)
        sc[:, :, :r, :c] += mask[:r, :c]
    sc = sc - sc.max(-1, keepdims=True)
    p = np.exp(sc)
    p = p / (p.sum(-1, keepdims=True) + 1e-10)
    a = (p @ vv).transpose(0, 2, 1, 3).reshape(B, S, H * hd)
    h = x + a @ W["wo"].T
    n2 = rmsnorm(h, W["n2"], eps)
    g = n2 @ W["w1"].T
    g = g / (1.0 + np.exp(-g)) * (n2 @ W["w3"].T)
    return h + g @ W["w2"].T


def close(got, ref, what, tol=TOL):
    ref = np.asarray(ref, dtype=np.float64)
    scale = np.sqrt((ref ** 2).mean()) + np.abs(ref)
    err = np.abs(got.astype(np.float64) - ref)
    bad = err > tol * scale
    assert np.isfinite(got).all(), what
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} beyond tol; worst {float((err / scale).max()):.2e}"
    return float((err / scale).max())


def as_array(t):
    """Writable numpy view of a host fp32 Tensor's data."""
    c = t.contents
    shape = tuple(c.shape[i] for i in range(c.ndim))
    return np.ctypeslib.as_array(c.data, shape=(int(c.size),)).reshape(shape)


def causal(S, L):
    vis = (L - S) + np.arange(S)[:, None]
    return np.where(np.arange(L)[None, :] <= vis, 0.0, -np.inf).astype(np.float32)


@pytest.mark.parametrize("qname", ["q8", "q4"])
def test_block_on_device_matches_reference(qname):
    L = voxq.lib()
    os.environ["VOXCPM_QUANT"] = qname
    L.tensor_cuda_shutdown()
    assert L.tensor_cuda_init() == 0
    rng = np.random.default_rng(11)
    B, D, H, KVH, hd, F, eps = 1, 256, 4, 2, 64, 512, 1e-6
    W = {"wq": exact_weight(rng, H * hd, D, qname), "wk": exact_weight(rng, KVH * hd, D, qname),
         "wv": exact_weight(rng, KVH * hd, D, qname), "wo": exact_weight(rng, D, H * hd, qname),
         "w1": exact_weight(rng, F, D, qname), "w2": exact_weight(rng, D, F, qname),
         "w3": exact_weight(rng, F, D, qname),
         "n1": (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32),
         "n2": (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)}
    keep = []
    try:
        T = {k: voxq.host_tensor(W[k]) for k in W}
        keep += list(T.values())
        for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3"):
            voxq.check(L.tensor_to_cuda(T[k]), "tensor_to_cuda")
        n1 = voxq.RmsNormDesc(T["n1"], eps)
        n2 = voxq.RmsNormDesc(T["n2"], eps)
        at = voxq.AttentionDesc(T["wq"], T["wk"], T["wv"], T["wo"], D, H, KVH, hd)
        ff = voxq.SwigluDesc(T["w1"], T["w2"], T["w3"], D, F)
        bd = voxq.BlockDesc(C.pointer(n1), C.pointer(at), C.pointer(n2), C.pointer(ff))
        positions = 96
        inv = 10000.0 ** (-np.arange(hd // 2) * 2.0 / hd)
        ang = np.arange(positions)[:, None] * inv[None, :]
        freqs_np = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
        freqs = voxq.host_tensor(freqs_np)
        keep.append(freqs)

        def run(S, pos, ck, cv, ref_ck, ref_cv, use_mask, use_freqs, what):
            x_np = rng.standard_normal((B, S, D)).astype(np.float32)
            x, out = voxq.host_tensor(x_np), voxq.host_tensor(np.zeros((B, S, D), np.float32))
            mask_np = causal(S, pos + S) if use_mask else None
            mask = voxq.host_tensor(mask_np) if use_mask else None
            try:
                r = L.voxq_transformer_block_forward(C.byref(bd), x, ck, cv, mask, freqs if use_freqs else None,
                                                     pos, out)
                assert r == 0, f"{what}: error {r}"
                got = voxq.host_tensor_view(out)
            finally:
                for t in (x, out) + ((mask,) if use_mask else ()):
                    voxq.free_tensor(t)
            ref = block_ref(x_np, W, ref_ck, ref_cv, mask_np, freqs_np if use_freqs else None, pos, H, KVH, hd, eps)
            e = close(got, ref, what)
            e2 = close(as_array(ck)[:, :, pos:pos + S], ref_ck[:, :, pos:pos + S], what + " (cache K rows)")
            close(as_array(cv)[:, :, pos:pos + S], ref_cv[:, :, pos:pos + S], what + " (cache V rows)")
            return e, e2

        def cache(max_seq):
            ck = voxq.host_tensor(np.zeros((B, KVH, max_seq, hd), np.float32))
            cv = voxq.host_tensor(np.zeros((B, KVH, max_seq, hd), np.float32))
            keep.extend([ck, cv])
            return ck, cv, np.zeros((B, KVH, max_seq, hd)), np.zeros((B, KVH, max_seq, hd))

        # DiT-style: a fresh cache filled whole, no mask, no RoPE (GEMV and GEMM projections); the
        # same call repeated with new inputs is captured into a CUDA graph on its second sighting
        # and replayed from then on
        for S in (5, 9):
            ck, cv, rk, rv = cache(S)
            for rep in range(4):
                run(S, 0, ck, cv, rk, rv, False, False, f"fill S={S} (call {rep + 1})")
        # prefill with a causal mask and RoPE into a longer cache, then decode steps
        ck, cv, rk, rv = cache(48)
        run(16, 0, ck, cv, rk, rv, True, True, "prefill S=16")
        for pos in (16, 17, 18):
            run(1, pos, ck, cv, rk, rv, False, True, f"decode pos={pos}")
        # the host cache changed behind the library: the mirror must re-read it
        hk = as_array(ck)
        hk[0, 0, 18, :] += 0.5
        rk[0, 0, 18, :] = hk[0, 0, 18, :]
        hk[0, 1, 3, :] -= 0.25  # a row the last-row check alone would miss is re-read with it
        rk[0, 1, 3, :] = hk[0, 1, 3, :]
        run(1, 19, ck, cv, rk, rv, False, True, "decode after host change")
        # a two-token continuation with its causal mask
        run(2, 20, ck, cv, rk, rv, True, True, "continuation S=2")
        # restart at pos 0 on the same cache
        rk[:] = 0.0
        rv[:] = 0.0
        run(3, 0, ck, cv, rk, rv, True, True, "restart S=3")
        # enough query rows (seq x heads per kv head >= 64) for the tiled attention kernel: a fill, and a
        # causal prefill with RoPE followed by a two-row continuation over more than one key tile
        ck2, cv2, rk2, rv2 = cache(40)
        run(40, 0, ck2, cv2, rk2, rv2, False, False, "fill S=40 (tiled attention)")
        ck3, cv3, rk3, rv3 = cache(96)
        run(36, 0, ck3, cv3, rk3, rv3, True, True, "prefill S=36 (tiled attention)")
        run(32, 36, ck3, cv3, rk3, rv3, True, True, "continuation S=32 over 68 > 2 key tiles")
        # a continuation of a long cache with few query tiles: the keys are split over several
        # CTAs and the splits combined (the RALM's per-patch call late in an utterance); the
        # earlier rows come from the host cache (a fresh mirror); the second call at the same
        # position passes an equal mask (its device copy is reused), the third a new one
        ck4, cv4, rk4, rv4 = cache(2304)
        for arr, ref in ((as_array(ck4), rk4), (as_array(cv4), rv4)):
            arr[:, :, :2048] = rng.standard_normal((B, KVH, 2048, hd)).astype(np.float32)
            ref[:, :, :2048] = arr[:, :, :2048]
        run(64, 2048, ck4, cv4, rk4, rv4, True, False, "continuation S=64 at pos 2048 (key splits)")
        run(64, 2048, ck4, cv4, rk4, rv4, True, False, "again at pos 2048 (mask reused)")
        run(64, 2112, ck4, cv4, rk4, rv4, True, False, "continuation S=64 at pos 2112 (key splits)")
        assert voxq.lib().voxq_device_error(1) == 0
    finally:
        for t in keep:
            voxq.free_tensor(t)
        L.voxq_block_cache_clear()
        L.tensor_cuda_shutdown()
        os.environ.pop("VOXCPM_QUANT", None)


def test_attention_at_the_engine_head_shape():
    """The engine's attention shape (head_dim 128, 16 query heads over 2 kv
    heads, so a CTA's 64 query vectors are 8 rows x 8 heads), through the
    tensor-core attention (the default) or, in the child-process test below,
    the CUDA-core kernel.  Calls of at most 8 rows project on the fp32 GEMV,
    so they are held to the block's 1e-3 rule: an 8-row fill (exactly the 64
    query vectors of one CTA) and an 8-row continuation of a 1024-row cache
    (keys split over CTAs) whose mask hides the first 40 keys of every row (a
    whole key tile with no visible key, then a partly visible one).  Larger
    calls project on the fp16 tensor-core GEMM and take the library's GEMM
    rule, 5e-3: a LocDiT-style fill of both CFG branches (B = 2, 201 rows, no
    mask; repeated, so the second call is captured into a CUDA graph and the
    third replays it), a causal prefill with RoPE, and a 64-row continuation
    with the same hidden keys."""
    L = voxq.lib()
    os.environ["VOXCPM_QUANT"] = "q8"
    L.tensor_cuda_shutdown()
    assert L.tensor_cuda_init() == 0
    rng = np.random.default_rng(29)
    D, H, KVH, hd, F, eps = 256, 16, 2, 128, 256, 1e-6
    W = {"wq": exact_weight(rng, H * hd, D, "q8"), "wk": exact_weight(rng, KVH * hd, D, "q8"),
         "wv": exact_weight(rng, KVH * hd, D, "q8"), "wo": exact_weight(rng, D, H * hd, "q8"),
         "w1": exact_weight(rng, F, D, "q8"), "w2": exact_weight(rng, D, F, "q8"),
         "w3": exact_weight(rng, F, D, "q8"),
         "n1": (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32),
         "n2": (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)}
    keep = []
    try:
        T = {k: voxq.host_tensor(W[k]) for k in W}
        keep += list(T.values())
        for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3"):
            voxq.check(L.tensor_to_cuda(T[k]), "tensor_to_cuda")
        n1 = voxq.RmsNormDesc(T["n1"], eps)
        n2 = voxq.RmsNormDesc(T["n2"], eps)
        at = voxq.AttentionDesc(T["wq"], T["wk"], T["wv"], T["wo"], D, H, KVH, hd)
        ff = voxq.SwigluDesc(T["w1"], T["w2"], T["w3"], D, F)
        bd = voxq.BlockDesc(C.pointer(n1), C.pointer(at), C.pointer(n2), C.pointer(ff))
        positions = 64
        inv = 10000.0 ** (-np.arange(hd // 2) * 2.0 / hd)
        ang = np.arange(positions)[:, None] * inv[None, :]
        freqs_np = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
        freqs = voxq.host_tensor(freqs_np)
        keep.append(freqs)

        def cache(B, max_seq):
            ck = voxq.host_tensor(np.zeros((B, KVH, max_seq, hd), np.float32))
            cv = voxq.host_tensor(np.zeros((B, KVH, max_seq, hd), np.float32))
            keep.extend([ck, cv])
            return ck, cv, np.zeros((B, KVH, max_seq, hd)), np.zeros((B, KVH, max_seq, hd))

        def run(B, S, pos, c, mask_np, use_freqs, what, tol=TOL):
            ck, cv, ref_ck, ref_cv = c
            x_np = rng.standard_normal((B, S, D)).astype(np.float32)
            x, out = voxq.host_tensor(x_np), voxq.host_tensor(np.zeros((B, S, D), np.float32))
            mask = voxq.host_tensor(mask_np) if mask_np is not None else None
            try:
                r = L.voxq_transformer_block_forward(C.byref(bd), x, ck, cv, mask, freqs if use_freqs else None,
                                                     pos, out)
                assert r == 0, f"{what}: error {r}"
                got = voxq.host_tensor_view(out)
            finally:
                for t_ in (x, out) + ((mask,) if mask is not None else ()):
                    voxq.free_tensor(t_)
            ref = block_ref(x_np, W, ref_ck, ref_cv, mask_np, freqs_np if use_freqs else None, pos, H, KVH, hd,
                            eps)
            close(got, ref, what, tol)
            close(as_array(ck)[:, :, pos:pos + S], ref_ck[:, :, pos:pos + S], what + " (cache K rows)", tol)

        gemm_tol = 5e-3  # more than 8 rows: projections on fp16 tensor cores
        c = cache(1, 8)
        run(1, 8, 0, c, None, False, "fill S=8 (64 query vectors)")
        c = cache(2, 201)
        for rep in range(3):
            run(2, 201, 0, c, None, False, f"fill B=2 S=201 (call {rep + 1})", gemm_tol)
        c = cache(1, 64)
        run(1, 40, 0, c, causal(40, 40), True, "prefill S=40", gemm_tol)
        c = cache(1, 1152)
        for arr, ref in ((as_array(c[0]), c[2]), (as_array(c[1]), c[3])):
            arr[:, :, :1024] = rng.standard_normal((1, KVH, 1024, hd)).astype(np.float32)
            ref[:, :, :1024] = arr[:, :, :1024]
        m = causal(8, 1032)
        m[:, :40] = -np.inf
        run(1, 8, 1024, c, m, False, "continuation S=8 at pos 1024, first 40 keys hidden (key splits)")
        m = causal(64, 1096)
        m[:, :40] = -np.inf
        run(1, 64, 1032, c, m, False, "continuation S=64 at pos 1032, first 40 keys hidden (key splits)",
            gemm_tol)
        assert voxq.lib().voxq_device_error(1) == 0
    finally:
        for t_ in keep:
            voxq.free_tensor(t_)
        L.voxq_block_cache_clear()
        L.tensor_cuda_shutdown()
        os.environ.pop("VOXCPM_QUANT", None)


def test_cuda_core_attention_in_child_process():
    """VOXQ_ATTN_MMA=0 (read once per process) selects the CUDA-core tiled
    attention kernel in place of the tensor-core one: the attention cases of
    this file run again in a child process with it set."""
    env = dict(os.environ, VOXQ_ATTN_MMA="0")
    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        os.path.join(here, "test_gpu_block.py"), "-k", "matches_reference or engine_head_shape"],
                       env=env, cwd=os.path.dirname(here), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "5 passed" in r.stdout, r.stdout[-2000:]


@pytest.mark.parametrize("qname", ["q8", "q4"])
def test_locenc_on_device_matches_reference(qname):
    """voxq_locenc_forward against a float64 restatement of loc_enc_forward
    (src/loc_enc.c:19-190): in_proj + bias, [special; P patches] per step, the
    layers over all T (P + 1) tokens (bidirectional, no RoPE, fresh cache at
    pos 0), each step's first token, output RMSNorm.  T = 2 takes the per-row
    attention kernel, T = 13 the tiled one.  Rule: 5e-3 of scale (two chained
    layers of fp16 tensor-core projections; one block alone meets 1e-3)."""
    L = voxq.lib()
    os.environ["VOXCPM_QUANT"] = qname
    L.tensor_cuda_shutdown()
    assert L.tensor_cuda_init() == 0
    rng = np.random.default_rng(23)
    D, H, KVH, hd, FF, eps, Fd, P, NL = 256, 4, 2, 64, 512, 1e-6, 64, 4, 2
    layers = []
    for _ in range(NL):
        layers.append({"wq": exact_weight(rng, H * hd, D, qname), "wk": exact_weight(rng, KVH * hd, D, qname),
                       "wv": exact_weight(rng, KVH * hd, D, qname), "wo": exact_weight(rng, D, H * hd, qname),
                       "w1": exact_weight(rng, FF, D, qname), "w2": exact_weight(rng, D, FF, qname),
                       "w3": exact_weight(rng, FF, D, qname),
                       "n1": (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32),
                       "n2": (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)})
    win = exact_weight(rng, D, Fd, qname)
    b_in = (0.02 * rng.standard_normal(D)).astype(np.float32)
    special = (0.02 * rng.standard_normal(D)).astype(np.float32)
    wn = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    keep, descs = [], []
    try:
        blocks = (voxq.BlockDesc * NL)()
        for l, W in enumerate(layers):
            T_ = {k: voxq.host_tensor(W[k]) for k in W}
            keep += list(T_.values())
            for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3"):
                voxq.check(L.tensor_to_cuda(T_[k]), "tensor_to_cuda")
            n1, n2 = voxq.RmsNormDesc(T_["n1"], eps), voxq.RmsNormDesc(T_["n2"], eps)
            at = voxq.AttentionDesc(T_["wq"], T_["wk"], T_["wv"], T_["wo"], D, H, KVH, hd)
            ff = voxq.SwigluDesc(T_["w1"], T_["w2"], T_["w3"], D, FF)
            descs += [n1, n2, at, ff]
            blocks[l] = voxq.BlockDesc(C.pointer(n1), C.pointer(at), C.pointer(n2), C.pointer(ff))
        tw, tb = voxq.host_tensor(win), voxq.host_tensor(b_in)
        ts = voxq.host_tensor(special.reshape(1, 1, 1, D))
        tn = voxq.host_tensor(wn)
        keep += [tw, tb, ts, tn]
        voxq.check(L.tensor_to_cuda(tw), "tensor_to_cuda")
        on = voxq.RmsNormDesc(tn, eps)
        enc = voxq.LocEncDesc(tw, tb, ts, C.cast(blocks, C.POINTER(voxq.BlockDesc)), NL, C.pointer(on), D, P)
        for T in (2, 13):
            feats = rng.standard_normal((1, T, P, Fd)).astype(np.float32)
            tf = voxq.host_tensor(feats)
            to = voxq.host_tensor(np.zeros((1, T, D), np.float32))
            try:
                assert L.voxq_locenc_forward(C.byref(enc), tf, to) == 0
                got = voxq.host_tensor_view(to)
            finally:
                voxq.free_tensor(tf)
                voxq.free_tensor(to)
            proj = feats.reshape(T * P, Fd).astype(np.float64) @ win.T.astype(np.float64) + b_in
            x = np.concatenate([np.broadcast_to(special, (T, 1, D)), proj.reshape(T, P, D)], 1)
            x = x.reshape(1, T * (P + 1), D)
            S = T * (P + 1)
            for W in layers:
                ck, cv = np.zeros((1, KVH, S, hd)), np.zeros((1, KVH, S, hd))
                x = block_ref(x, W, ck, cv, None, None, 0, H, KVH, hd, eps)
            ref = rmsnorm(x.reshape(T, P + 1, D)[:, 0][None], wn, eps)
            # two chained layers whose projections (more than 8 rows) run on fp16 tensor cores:
            # the library's GEMM rule, 5e-3, rather than the single block's 1e-3
            close(got, ref, f"locenc {qname} T={T}", tol=5e-3)
        assert L.voxq_device_error(1) == 0
    finally:
        for t in keep:
            voxq.free_tensor(t)
        L.voxq_block_cache_clear()
        L.tensor_cuda_shutdown()
        os.environ.pop("VOXCPM_QUANT", None)


def test_block_declines_what_it_does_not_take():
    """Unquantized weights, device operands or an uninitialised library: VOXCPM_ERR_CUDA_NOT_FOUND,
    so the engine runs its own host code."""
    L = voxq.lib()
    os.environ.pop("VOXCPM_QUANT", None)
    L.tensor_cuda_shutdown()
    assert L.tensor_cuda_init() == 0
    D, H, KVH, hd, F = 64, 2, 1, 32, 128
    rng = np.random.default_rng(3)
    keep = []
    try:
        T = {k: voxq.host_tensor(rng.standard_normal(s).astype(np.float32) * 0.05) for k, s in
             (("wq", (H * hd, D)), ("wk", (KVH * hd, D)), ("wv", (KVH * hd, D)), ("wo", (D, H * hd)),
              ("w1", (F, D)), ("w2", (D, F)), ("w3", (F, D)), ("n1", (D,)), ("n2", (D,)))}
        keep += list(T.values())
        for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3"):
            voxq.check(L.tensor_to_cuda(T[k]), "tensor_to_cuda")  # dense fp32 device weights
        n1, n2 = voxq.RmsNormDesc(T["n1"], 1e-6), voxq.RmsNormDesc(T["n2"], 1e-6)
        at = voxq.AttentionDesc(T["wq"], T["wk"], T["wv"], T["wo"], D, H, KVH, hd)
        ff = voxq.SwigluDesc(T["w1"], T["w2"], T["w3"], D, F)
        bd = voxq.BlockDesc(C.pointer(n1), C.pointer(at), C.pointer(n2), C.pointer(ff))
        x = voxq.host_tensor(np.zeros((1, 3, D), np.float32))
        out = voxq.host_tensor(np.zeros((1, 3, D), np.float32))
        ck = voxq.host_tensor(np.zeros((1, KVH, 3, hd), np.float32))
        cv = voxq.host_tensor(np.zeros((1, KVH, 3, hd), np.float32))
        keep += [x, out, ck, cv]
        assert L.voxq_transformer_block_forward(C.byref(bd), x, ck, cv, None, None, 0, out) == voxq.CUDA_NOT_FOUND
        L.tensor_cuda_shutdown()
        assert L.voxq_transformer_block_forward(C.byref(bd), x, ck, cv, None, None, 0, out) == voxq.CUDA_NOT_FOUND
    finally:
        L.tensor_cuda_init()
        for t in keep:
            voxq.free_tensor(t)
        L.tensor_cuda_shutdown()
