"""Structural graph cache of the token loop (vkllm_models_llama2_build_graph / vkllm_graph_free).

The reference loop rebuilds the whole graph every token (tests/vkllm_test_infer_gguf.c:181-272). With
the cache, vkllm_graph_free keeps the nodes of a model-built graph and the next build with the same
model, batch and token count reuses them, rewriting the position-dependent fields. These tests check
that a build from the cache is indistinguishable from a fresh build (every node's name, op, dtype,
shapes, strides, byte size, params and sources, and the KV-cache tensors' sources and offsets), that
the token loop produces bit-identical tokens and logits with the cache on and off in both execution
modes (across the key count where the attention product changes kernel, Lk == head_dim), that the
context's allocation counters advance the same, and the lifetime cases: two live graphs of one
structure, a graph whose node list the caller changed, and a model freed while its graph lives."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_PROMPT = 32


def _stats(ctx):
    base = ctx.ptr.value + 3 * C.sizeof(C.c_void_p)  # appname, device, runtime, then stats
    return C.c_int.from_address(base).value, C.c_int.from_address(base + 4).value


def _build(vk, ctx, model, toks, offset):
    l = vk.lib()
    inp = vk.tensor_new(ctx, "input_toks", (1, 1, 1, len(toks)), vk.U32, mapped=True)
    g = C.POINTER(vk.Graph)()
    vk.check(l.vkllm_graph_new(ctx.ptr, C.byref(g)), "graph_new")
    vk.check(l.vkllm_models_llama2_build_graph(ctx.ptr, C.byref(model.m), inp, g, offset), "build_graph")
    return g


def _free(vk, ctx, g):
    vk.lib().vkllm_graph_free(ctx.ptr, g)


def _ext_label(p):
    return ("ext", C.cast(p, C.POINTER(C.c_char * 128)).contents.value)


def _dump(vk, model, g):
    """Every node as (name, op, dtype, shapes, strides, bytes, is_ref, mapped, params[0:12], sources),
    sources as graph indices or the names of tensors outside the graph; plus, per layer, the
    KV-cache tensors' (source index, params offset)."""
    nodes = g.contents.nodes.contents
    arr = C.cast(nodes.data, C.POINTER(C.c_void_p))
    ptrs = [arr[i] for i in range(nodes.used_n)]
    index = {p: i for i, p in enumerate(ptrs)}
    out = []
    for p in ptrs:
        t = C.cast(p, vk.PT).contents
        params = bytes((C.c_ubyte * 12).from_address(p + C.sizeof(vk.Tensor)))
        srcs = tuple(None if not s else (("node", index[s]) if s in index else _ext_label(s)) for s in t.srcs)
        out.append((t.name, t.op, t.dtype, tuple(t.shapes), tuple(t.strides), t.bytes, t.data.is_ref,
                    t.data.mapped, params, srcs))
    kv = C.cast(model.m.weights.kvcache, C.POINTER(vk.KVCache)).contents
    caches = []
    for arr_p in (kv.kcaches, kv.vcaches):
        a = arr_p.contents
        items = C.cast(a.data, C.POINTER(C.c_void_p))
        for i in range(a.used_n):
            t = C.cast(items[i], vk.PT).contents
            off = C.c_uint32.from_address(items[i] + C.sizeof(vk.Tensor)).value
            caches.append((index.get(t.srcs[0]), off))
    return out, caches


def test_cached_build_matches_fresh_build(vk, ctx, tiny_gguf, monkeypatch):
    path, _ = tiny_gguf
    monkeypatch.setenv("VKLLM_B200_GRAPH_CACHE", "0")
    ctx_off = vk.Context(0)
    monkeypatch.delenv("VKLLM_B200_GRAPH_CACHE")
    m_on, m_off = vk.Model(ctx).load(path), vk.Model(ctx_off).load(path)
    try:
        for S in (1, 5):
            toks = list(range(3, 3 + S))
            g = _build(vk, ctx, m_on, toks, 2)  # fresh: registers the structure
            _free(vk, ctx, g)
            for offset in (7, 47, 48, 120):  # Lk crosses head_dim (48) for S = 1
                g_on = _build(vk, ctx, m_on, toks, offset)
                g_off = _build(vk, ctx_off, m_off, toks, offset)
                try:
                    d_on, c_on = _dump(vk, m_on, g_on)
                    d_off, c_off = _dump(vk, m_off, g_off)
                    assert len(d_on) == len(d_off)
                    for i, (a, b) in enumerate(zip(d_on, d_off)):
                        assert a == b, (S, offset, i, a, b)
                    assert c_on == c_off, (S, offset)
                    assert all(off == offset for _, off in c_on)
                finally:
                    _free(vk, ctx, g_on)
                    _free(vk, ctx_off, g_off)
    finally:
        m_on.free()
        m_off.free()
        ctx_off.close()


@pytest.mark.parametrize("strict", [True, False], ids=["strict", "fused"])
def test_token_loop_identical_with_and_without_cache(vk, ctx, tiny_gguf, strict, monkeypatch):
    import gen_gguf

    path, _ = tiny_gguf
    prompt = gen_gguf.prompt(7, N_PROMPT)
    monkeypatch.setenv("VKLLM_B200_GRAPH_CACHE", "0")
    ctx_off = vk.Context(0)
    monkeypatch.delenv("VKLLM_B200_GRAPH_CACHE")
    mode = vk.EXEC_STRICT if strict else vk.EXEC_FUSED
    runs = []
    try:
        for c in (ctx, ctx_off):
            c.set_exec_mode(mode)
            m = vk.Model(c).load(path)
            try:
                s0 = _stats(c)
                logits = []
                toks = m.generate(prompt, 24, logits)  # decode keys 33..56: Lk == hd = 48 inside
                s1 = _stats(c)
            finally:
                m.free()
            runs.append((toks, np.stack(logits), (s1[0] - s0[0], s1[1] - s0[1])))
    finally:
        ctx.set_exec_mode(vk.EXEC_FUSED)
        ctx_off.close()
    (t_on, l_on, st_on), (t_off, l_off, st_off) = runs
    assert t_on == t_off
    assert np.array_equal(l_on.view(np.uint16), l_off.view(np.uint16))
    assert st_on == st_off, (st_on, st_off)


def test_cache_lifetimes(vk, ctx, tiny_gguf):
    path, _ = tiny_gguf
    l = vk.lib()
    ctx.set_graph_cache(True)

    def run(g):
        vk.check(l.vkllm_graph_init(ctx.ptr, g), "init")
        inp = g.contents.nodes.contents
        t0 = C.cast(C.cast(inp.data, C.POINTER(C.c_void_p))[0], vk.PT)
        n = t0.contents.shapes[3]
        C.memmove(t0.contents.data.host, (C.c_uint32 * n)(*range(5, 5 + n)), 4 * n)
        vk.check(l.vkllm_graph_run(ctx.ptr, g), "run")
        out = g.contents.output_node.contents
        return C.cast(out.data.host, C.POINTER(C.c_uint32))[out.shapes[2] - 1]

    m = vk.Model(ctx).load(path)
    try:
        ref = []
        for off in range(4):  # reference tokens from fresh builds (cache off)
            ctx.set_graph_cache(False)
            g = _build(vk, ctx, m, [9], off)
            ref.append(run(g))
            _free(vk, ctx, g)
        ctx.set_graph_cache(True)
        # two live graphs of one structure: the second is built fresh and freed normally
        g1 = _build(vk, ctx, m, [9], 0)
        g2 = _build(vk, ctx, m, [9], 1)
        assert [run(g1), run(g2)] == ref[:2]
        _free(vk, ctx, g2)
        _free(vk, ctx, g1)
        g3 = _build(vk, ctx, m, [9], 2)  # from the cache
        assert run(g3) == ref[2]
        # the caller adds a node: the graph frees everything itself and the entry goes
        extra = vk.tensor_new(ctx, "extra", (1, 1, 1, 4), vk.U32)
        vk.check(l.vkllm_graph_add_node(ctx.ptr, g3, extra), "add_node")
        _free(vk, ctx, g3)
        g4 = _build(vk, ctx, m, [9], 3)
        assert run(g4) == ref[3]
        _free(vk, ctx, g4)
        # a model freed while its graph lives: the graph still frees its own nodes
        g5 = _build(vk, ctx, m, [9], 0)
        m.free()
        _free(vk, ctx, g5)
    finally:
        m.free()


def test_native_token_loop_matches_the_python_loop(vk, ctx, tiny_gguf):
    """vkllm_b200_token_loop (the reference loop's calls in native code) predicts what the same calls
    made one by one from Python predict, prefill included."""
    import gen_gguf

    path, _ = tiny_gguf
    prompt = gen_gguf.prompt(9, 12)
    m = vk.Model(ctx).load(path)
    try:
        py = m.generate(prompt, 20)
        native, host_us = m.token_loop(prompt, 0, 20)
    finally:
        m.free()
    assert native == py
    assert host_us > 0
