"""Generates tests/golden/ref_ops.npz: seeded inputs and the outputs of the reference's own test-side
CPU references, restated in numpy. They pin the oracle (tests/test_oracle.py).

vkllm.c stores no golden vectors: each op test in its tests/ directory draws random inputs and
compares the Vulkan result with an in-file CPU function. Those functions define the expected
formulas, and this script restates them:

  matmul      tests/vkllm_test_op_matmul.c:33-165     (fp32 sum over k, optional SiLU, broadcast B/C)
  rmsnorm     tests/vkllm_test_op_rmsnorm.c:14-106    (x * g / sqrt(mean(x^2) + eps))
  rope        tests/vkllm_test_op_rope.c:17-94        (pair rotation, theta = (offset + h) / base^(2w/W))
  softmax     tests/vkllm_test_op_softmax.c:14-119    (masked w > h + offsets -> 0; max over unmasked)
  arg_max     tests/vkllm_test_op_arg_max.c:12-71     (first strict maximum)
  update_rows tests/vkllm_test_op_update_rows.c:75-122 (cache[:, :, off + h, :] = src[:, :, h, :])
  embedding   tests/vkllm_test_op_embedding.c:32-94   (out[h, :] = table[id_h, :])

Outputs are stored through the tests' fp32 -> fp16 conversion, which truncates the mantissa
(src/core/vkllm_common.h:157-186); `to_f16_trunc` restates it. Inputs come from
numpy.random.default_rng with fixed seeds (the reference's tests use unseeded rand()).

Run:  python tests/golden/make_golden.py   (rewrites ref_ops.npz next to this file)
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def to_f16_trunc(x):
    """The reference tests' fp32 -> fp16: exponent re-biased and clamped, mantissa truncated."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    sign = (u >> 31) & 1
    exp = ((u >> 23) & 0xFF).astype(np.int64)
    frac = u & 0x7FFFFF
    nan = (exp == 255) & (frac != 0)
    e = exp - 127
    he = np.where(e < -14, 0, np.where(e > 15, 31, e + 15))
    bits = (sign << 15) | (he.astype(np.uint32) << 10) | (frac >> 13)
    bits = np.where(nan, (sign << 15) | (31 << 10) | 1, bits)
    return bits.astype(np.uint16).view(np.float16)


def silu(v):
    return v / (1.0 + np.exp(-v))


def ref_matmul(a, b, transposed_b, act, out_f16=True):
    """C[b,c,i,j] = sum_k A[ba,ca,i,k] * B[bb,cb,(j,k) or (k,j)] with dims of size 1 broadcast."""
    B = max(a.shape[0], b.shape[0])
    Cc = max(a.shape[1], b.shape[1])
    M, K = a.shape[2], a.shape[3]
    N = b.shape[2] if transposed_b else b.shape[3]
    out = np.zeros((B, Cc, M, N), dtype=np.float32)
    af, bf = a.astype(np.float32), b.astype(np.float32)
    for bi in range(B):
        for ci in range(Cc):
            A = af[0 if a.shape[0] == 1 else bi, 0 if a.shape[1] == 1 else ci]
            Bm = bf[0 if b.shape[0] == 1 else bi, 0 if b.shape[1] == 1 else ci]
            r = A @ (Bm.T if transposed_b else Bm)
            out[bi, ci] = silu(r) if act else r
    return to_f16_trunc(out) if out_f16 else out


def ref_rmsnorm(x, g, eps):
    xf = x.astype(np.float32)
    rms = np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + np.float32(eps))
    return to_f16_trunc(xf / rms * g.reshape(1, 1, 1, -1))


def ref_rope(x, offset, base):
    B, Cc, H, W = x.shape
    xf = x.astype(np.float32)
    out = np.zeros(x.shape, dtype=np.float32)
    w = np.arange(W // 2, dtype=np.float32)
    for h in range(H):
        th = np.float32(offset + h) / np.power(np.float32(base), (2 * w) / np.float32(W))
        c, s = np.cos(th), np.sin(th)
        v0, v1 = xf[:, :, h, 0::2], xf[:, :, h, 1::2]
        out[:, :, h, 0::2] = c * v0 - s * v1
        out[:, :, h, 1::2] = s * v0 + c * v1
    return to_f16_trunc(out)


def ref_softmax(x, seq_mask, offsets):
    B, Cc, H, W = x.shape
    xf = x.astype(np.float32)
    out = np.zeros(x.shape, dtype=np.float32)
    for h in range(H):
        keep = np.ones(W, dtype=bool) if seq_mask <= 0 else (np.arange(W) <= h + offsets)
        row = xf[:, :, h, :]
        mx = np.max(np.where(keep, row, -np.inf), axis=-1, keepdims=True)
        e = np.where(keep, np.exp(row - mx), 0.0)
        out[:, :, h, :] = e / np.sum(e, axis=-1, keepdims=True)
    return to_f16_trunc(out)


def ref_arg_max(x):
    xf = x.astype(np.float32)
    B, Cc, H, W = x.shape
    out = np.zeros((B, Cc, H, 1), dtype=np.uint32)
    for b in range(B):
        for c in range(Cc):
            for h in range(H):
                best, bi = -np.inf, 0
                for w in range(W):
                    if xf[b, c, h, w] > best:
                        best, bi = xf[b, c, h, w], w
                out[b, c, h, 0] = bi
    return out


def ref_arg_max_shader(x):
    """src/shaders/vkllm_arg_max.comp:54-90: lane l scans w = l, l+32, ... keeping the first strict
    maximum (an empty lane keeps -FLT_MAX and its own index), then a 16/8/4/2/1 tree keeps the left
    operand unless the right one is strictly greater. It differs from the test's first maximum only
    on ties (quirk Q8)."""
    xf = x.astype(np.float32)
    B, Cc, H, W = x.shape
    out = np.zeros((B, Cc, H, 1), dtype=np.uint32)
    fmax = np.float32(np.finfo(np.float32).max)
    for b in range(B):
        for c in range(Cc):
            for h in range(H):
                vals = [(-fmax, l) if l >= W else (xf[b, c, h, l], l) for l in range(32)]
                for l in range(32):
                    for i in range(l + 32, W, 32):
                        if xf[b, c, h, i] > vals[l][0]:
                            vals[l] = (xf[b, c, h, i], i)
                step = 16
                while step > 0:
                    for l in range(step):
                        if vals[l + step][0] > vals[l][0]:
                            vals[l] = vals[l + step]
                    step //= 2
                out[b, c, h, 0] = vals[0][1]
    return out


def ref_update_rows(src, cache, off):
    out = cache.copy()
    out[:, :, off:off + src.shape[2], :] = src
    return out


def ref_embedding(ids, table, unk):
    idx = np.where(ids.reshape(-1) >= table.shape[2], unk, ids.reshape(-1))
    return table[0, 0, idx, :].reshape(1, 1, -1, table.shape[3])


def f16(rng, shape, lo=-1.0, hi=1.0):
    return rng.uniform(lo, hi, size=shape).astype(np.float32).astype(np.float16)


def main():
    rng = np.random.default_rng(20240611)
    g = {}
    # matmul families of tests/vkllm_test_op_matmul.c:179-286 at reduced sizes
    mm = [("gemv", (1, 1), (1, 1), 1, 1024, 256, True, 0),
          ("odd_t", (1, 1), (1, 1), 33, 259, 65, True, 0),
          ("odd_n", (1, 1), (1, 1), 33, 259, 65, False, 0),
          ("batch_t", (2, 2), (2, 2), 16, 64, 32, True, 0),
          ("batch_n", (2, 2), (2, 2), 16, 64, 32, False, 0),
          ("bcast_a", (1, 1), (4, 1), 8, 32, 16, True, 0),
          ("bcast_b", (1, 4), (1, 1), 8, 32, 16, False, 0),
          ("silu_t", (1, 1), (1, 1), 12, 96, 40, True, 1)]
    for name, (Ba, Ca), (Bb, Cb), M, K, N, tb, act in mm:
        a = f16(rng, (Ba, Ca, M, K))
        b = f16(rng, (Bb, Cb, N, K) if tb else (Bb, Cb, K, N))
        g[f"mm_{name}_a"], g[f"mm_{name}_b"] = a, b
        g[f"mm_{name}_meta"] = np.array([M, K, N, int(tb), act], dtype=np.int64)
        g[f"mm_{name}_out"] = ref_matmul(a, b, tb, act)
    # rmsnorm: fp16 input, fp32 gains (the model path), tests/vkllm_test_op_rmsnorm.c
    x = f16(rng, (1, 1, 11, 320), -2.0, 2.0)
    gw = rng.uniform(0.5, 1.5, size=320).astype(np.float32)
    g["rms_x"], g["rms_g"], g["rms_out"] = x, gw, ref_rmsnorm(x, gw, 1e-6)
    # rope on a contiguous [1, 4, 11, 32] and on the strided head view of [1, 1, 11, 128]
    x = f16(rng, (1, 4, 11, 32))
    g["rope_x"], g["rope_out"] = x, ref_rope(x, 5, 10000.0)
    flat = f16(rng, (1, 1, 11, 128))
    g["rope_flat"] = flat
    g["rope_view_out"] = ref_rope(flat.reshape(1, 11, 4, 32).transpose(0, 2, 1, 3), 3, 10000.0)
    # softmax widths of tests/vkllm_test_op_softmax.c:121-145, masked and unmasked
    for W, mask, off in ((64, 0, 0), (130, 1, 0), (96, 1, 40)):
        x = f16(rng, (1, 2, 4, W), -4.0, 4.0)
        g[f"sm_{W}_{mask}_{off}_x"] = x
        g[f"sm_{W}_{mask}_{off}_out"] = ref_softmax(x, mask, off)
    # arg_max with planted ties (the first maximum wins)
    x = f16(rng, (1, 1, 3, 1000))
    x[0, 0, 0, 17] = x[0, 0, 0, 900] = np.float16(3.0)
    x[0, 0, 1, 5] = x[0, 0, 1, 6] = np.float16(2.5)
    g["am_x"], g["am_out"], g["am_out_shader"] = x, ref_arg_max(x), ref_arg_max_shader(x)
    # update_rows with an offset, into a zeroed cache
    src = f16(rng, (1, 4, 3, 16))
    cache = np.zeros((1, 4, 32, 16), dtype=np.float16)
    g["ur_src"], g["ur_cache"], g["ur_out"] = src, cache, ref_update_rows(src, cache, 7)
    # embedding with an out-of-vocabulary id mapped to unk
    table = f16(rng, (1, 1, 50, 32))
    ids = np.array([3, 0, 49, 50, 12, 77, 3, 1], dtype=np.uint32).reshape(1, 1, 1, 8)
    g["emb_table"], g["emb_ids"], g["emb_out"] = table, ids, ref_embedding(ids, table, 2)
    np.savez_compressed(os.path.join(HERE, "ref_ops.npz"), **g)
    print("wrote", os.path.join(HERE, "ref_ops.npz"), sum(v.nbytes for v in g.values()), "bytes")


if __name__ == "__main__":
    main()
