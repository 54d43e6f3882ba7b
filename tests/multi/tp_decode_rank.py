"""One rank of a tensor-parallel decode run (launched by tests/test_tp_gpu.py under torchrun, one
process per GPU): builds shard RANK of WORLD of a random model, connects the exchange (EXCHANGE:
"peer", the peer-memory exchange inside the persistent kernel, handles gathered over gloo; or "nccl",
the per-op kernels with NCCL collectives, the unique id gathered over gloo), decodes a prompt token
by token and then greedily on the engine, and writes its tokens and its vocabulary shard of every
generated step's logits to OUT/rank<r>.npz. Usage: tp_decode_rank.py OUT [EXCHANGE]."""
import os
import sys

import numpy as np
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "vkllm.c_b200"))
import vkllm_b200 as vk  # noqa: E402

CFG = dict(block_count=2, context_length=64, embedding_length=256, head_count=4, ffn_length=512, vocab_size=1000,
           rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)
SEED, PROMPT, N_GEN = 7, [11, 22, 33, 44, 55], 8


def main(out_dir, exchange):
    import ctypes as C

    dist.init_process_group("gloo", init_method="env://")
    rank, world = dist.get_rank(), dist.get_world_size()
    l = vk.lib()
    with vk.Context(rank) as ctx:
        model = vk.Model(ctx).init_random_tp(CFG, SEED, rank, world)

        def gather(b):
            got = [None] * world
            dist.all_gather_object(got, b)
            return got

        try:
            if exchange == "nccl":
                model.tp_connect_nccl(gather)
            else:
                model.tp_connect(gather)
            Vl = CFG["vocab_size"] // world
            logits = []
            for i, t in enumerate(PROMPT):  # teacher-forced prompt, one token per step
                vk.check(l.vkllm_b200_engine_set_state(ctx.ptr, C.byref(model.m), t, i), "set_state")
                vk.check(l.vkllm_b200_engine_decode_steps(ctx.ptr, C.byref(model.m), 1), "decode")
            persistent = l.vkllm_b200_engine_is_persistent(ctx.ptr, C.byref(model.m))
            assert bool(persistent) == (exchange != "nccl"), (exchange, persistent)
            buf = np.zeros(Vl, dtype=np.uint16)
            vk.check(l.vkllm_b200_engine_read_logits(ctx.ptr, C.byref(model.m), buf.ctypes.data, Vl), "logits")
            logits.append(buf.view(np.float16).copy())
            for _ in range(N_GEN - 1):
                vk.check(l.vkllm_b200_engine_decode_steps(ctx.ptr, C.byref(model.m), 1), "decode")
                vk.check(l.vkllm_b200_engine_read_logits(ctx.ptr, C.byref(model.m), buf.ctypes.data, Vl), "logits")
                logits.append(buf.view(np.float16).copy())
            toks = np.zeros(N_GEN, dtype=np.uint32)
            vk.check(l.vkllm_b200_engine_read_tokens(ctx.ptr, C.byref(model.m), toks.ctypes.data, N_GEN), "tokens")
            np.savez(os.path.join(out_dir, f"rank{rank}.npz"), toks=toks, logits=np.stack(logits))
        finally:
            dist.barrier()
            model.free()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "peer")
