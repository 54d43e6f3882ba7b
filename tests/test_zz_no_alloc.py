"""The allocation-free decode attention entry point (vkllm_b200_attention_decode_noalloc), for callers
that cannot allocate device memory (during stream capture, under a fixed memory budget, on
real-time paths). It is checked against two things that compute the same result: the CPU oracle's
restatement of the reference's three attention nodes (scores MATMUL with scale 1/sqrt(hd), SOFTMAX
with the causal mask at offset n_keys-1, probs.V MATMUL, each rounded to fp16), and the existing
entry points that run those nodes on the GPU (vkllm_op_matmul, vkllm_op_softmax). Two calls run in
a row (the second with a different key count, so stale scratch from the first call would show).
The kernels behind it contain no waits, so a fault would surface as a CUDA error when the stream is
synchronised by the read-back. This file sorts last so that a run that stops at the first failure
has already run every other test; it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(4242)


def close(gpu, ref, rel=2e-3):
    g = np.asarray(gpu, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(r).max(), 1e-6)
    bad = np.abs(g - r) > rel * np.abs(r) + rel * scale
    assert not bad.any(), f"{bad.sum()} of {bad.size} mismatches; max abs diff {np.abs(g - r).max()}"


def attention_via_oracle(orc, q, kc, vc, H, hd, n_keys):
    """The reference graph's attention nodes on the CPU (quirk Q1 included: at n_keys == hd the
    probs.V node reads V transposed, by the same shape predicate)."""
    ks = np.ascontiguousarray(kc[:, :, :n_keys, :])
    vs = np.ascontiguousarray(vc[:, :, :n_keys, :])
    scores = orc.matmul(q, ks, (1, H, 1, n_keys), 1.0 / np.sqrt(hd), 0)
    probs = orc.softmax(scores, 1, n_keys - 1)
    return orc.matmul(probs, vs, (1, H, 1, hd), 1.0, 0).reshape(H, hd)


def attention_via_ops(vk, ctx, Qt, Kt, Vt, H, hd, n_keys):
    """scores = Q . K[:n]^T * scale -> softmax -> probs . V[:n], through the existing op entry points."""
    lib = vk.lib()
    ext = (C.c_uint32 * 4)(1, H, n_keys, hd)
    Ks, Vs = vk.PT(), vk.PT()
    vk.check(lib.vkllm_tensor_slice0(ctx.ptr, Kt, ext, C.byref(Ks)), "slice0 k")
    vk.check(lib.vkllm_tensor_slice0(ctx.ptr, Vt, ext, C.byref(Vs)), "slice0 v")
    scale = 1.0 / np.sqrt(hd)
    sc = vk.tensor_new(ctx, "scores", (1, H, 1, n_keys), vk.F16, op=vk.OP_MATMUL, srcs=[Qt, Ks],
                       params=bytes(C.c_float(scale)) + bytes(C.c_int32(0)))
    vk.run_op(ctx, sc, "vkllm_op_matmul_init", "vkllm_op_matmul_run")
    pr = vk.tensor_new(ctx, "probs", (1, H, 1, n_keys), vk.F16, op=vk.OP_SOFTMAX, srcs=[sc],
                       params=bytes(C.c_int32(1)) + bytes(C.c_uint32(n_keys - 1)))
    vk.run_op(ctx, pr, "vkllm_op_softmax_init", "vkllm_op_softmax_run")
    out = vk.tensor_new(ctx, "attn", (1, H, 1, hd), vk.F16, op=vk.OP_MATMUL, srcs=[pr, Vs],
                        params=bytes(C.c_float(1.0)) + bytes(C.c_int32(0)))
    vk.run_op(ctx, out, "vkllm_op_matmul_init", "vkllm_op_matmul_run")
    res = vk.fetch(ctx, out).reshape(H, hd)
    for t in (out, pr, sc, Ks, Vs):
        vk.tensor_free(ctx, t)
    return res


@pytest.mark.parametrize("H,hd,rows,keys", [(6, 48, 256, (100, 37)), (32, 128, 1024, (777, 513)),
                                            (6, 48, 256, (48, 201))])
def test_noalloc_attention_matches_oracle_and_op_path(vk, ctx, orc, H, hd, rows, keys):
    lib = vk.lib()
    q = RNG.uniform(-1, 1, size=(1, H, 1, hd)).astype(np.float16)
    kc = RNG.uniform(-1, 1, size=(1, H, rows, hd)).astype(np.float16)
    vc = RNG.uniform(-1, 1, size=(1, H, rows, hd)).astype(np.float16)
    Qt = vk.tensor_new(ctx, "q", q.shape, vk.F16)
    Kt = vk.tensor_new(ctx, "k", kc.shape, vk.F16)
    Vt = vk.tensor_new(ctx, "v", vc.shape, vk.F16)
    Ot = vk.tensor_new(ctx, "o", (1, H, 1, hd), vk.F16)
    for t, a in ((Qt, q), (Kt, kc), (Vt, vc), (Ot, np.zeros((1, H, 1, hd), np.float16))):
        vk.put(ctx, t, a)
    try:
        for n_keys in keys:  # two calls in a row on the shared scratch
            ref = attention_via_ops(vk, ctx, Qt, Kt, Vt, H, hd, n_keys)
            err = lib.vkllm_b200_attention_decode_noalloc(Qt.contents.data.dev, Kt.contents.data.dev,
                                                          Vt.contents.data.dev, H, hd, rows, n_keys,
                                                          1.0 / np.sqrt(hd), Ot.contents.data.dev, ctx.stream)
            assert err == vk.OK
            got = vk.fetch(ctx, Ot).reshape(H, hd)  # same stream: ordered after the attention kernels
            close(got, ref)
            close(got, attention_via_oracle(orc, q, kc, vc, H, hd, n_keys))
    finally:
        for t in (Qt, Kt, Vt, Ot):
            vk.tensor_free(ctx, t)


def test_noalloc_attention_rejects_sizes_beyond_the_scratch(vk, ctx):
    lib = vk.lib()
    dummy = C.c_void_p(16)  # never dereferenced: the size check fails first
    assert lib.vkllm_b200_attention_decode_noalloc(dummy, dummy, dummy, 65, 128, 64, 1, 1.0, dummy, None) == vk.ARGS
    assert lib.vkllm_b200_attention_decode_noalloc(dummy, dummy, dummy, 64, 128, 8192, 1, 1.0, dummy, None) == vk.ARGS
    assert lib.vkllm_b200_attention_decode_noalloc(dummy, dummy, dummy, 8, 258, 64, 1, 1.0, dummy, None) == vk.ARGS
    assert lib.vkllm_b200_attention_decode_noalloc(dummy, dummy, dummy, 8, 128, 64, 65, 1.0, dummy, None) == vk.ARGS


def test_noalloc_attention_rejects_misaligned_caches(vk, ctx):
    """Cache rows are read 8 bytes at a time: a cache pointer off an 8-byte boundary (a sub-view of
    a larger fp16 buffer, say) is refused before any launch instead of faulting on the GPU."""
    lib = vk.lib()
    ok, odd2, odd1 = C.c_void_p(256), C.c_void_p(258), C.c_void_p(257)  # never dereferenced
    assert lib.vkllm_b200_attention_decode_noalloc(ok, odd2, ok, 8, 128, 64, 4, 1.0, ok, None) == vk.ARGS
    assert lib.vkllm_b200_attention_decode_noalloc(ok, ok, odd2, 8, 128, 64, 4, 1.0, ok, None) == vk.ARGS
    assert lib.vkllm_b200_attention_decode_noalloc(odd1, ok, ok, 8, 128, 64, 4, 1.0, ok, None) == vk.ARGS
    assert lib.vkllm_b200_attention_decode_noalloc(ok, ok, ok, 8, 128, 64, 4, 1.0, odd1, None) == vk.ARGS


def test_noalloc_attention_under_stream_capture(vk, ctx):
    """The use the entry point exists for: recorded into a CUDA graph by stream capture (where a device
    allocation is an error that invalidates the capture) and replayed. After one eager call (which
    resolves the scratch array's address), the captured call records without error, and its replays
    give the eager call's bits."""
    import torch

    lib = vk.lib()
    H, hd, rows, n = 8, 128, 512, 300
    g = torch.Generator(device="cuda").manual_seed(7)
    q = (torch.rand((H, hd), generator=g, device="cuda") * 2 - 1).half()
    kc = (torch.rand((H, rows, hd), generator=g, device="cuda") * 2 - 1).half()
    vc = (torch.rand((H, rows, hd), generator=g, device="cuda") * 2 - 1).half()
    out_eager = torch.zeros((H, hd), device="cuda", dtype=torch.float16)
    out_graph = torch.full((H, hd), float("nan"), device="cuda", dtype=torch.float16)
    scale = 1.0 / np.sqrt(hd)
    s = torch.cuda.Stream()

    def call(out):
        return lib.vkllm_b200_attention_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), H, hd, rows, n,
                                                       scale, out.data_ptr(), C.c_void_p(s.cuda_stream))

    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        assert call(out_eager) == vk.OK
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        err = call(out_graph)
    assert err == vk.OK
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_graph, out_eager)
    del graph
