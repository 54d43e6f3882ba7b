"""One rank of the CPU (gloo) check of the tensor-parallel weight layout: the rank asks the library
for its shard of each matrix kind (vkllm_b200_tp_shard), generates the shard's bits with the host
twin of the device generator (vkllm_b200_random_f16_host_shard, what init_random_tp writes on the
GPU), and all ranks gather them; rank 0 checks that the shards tile every unsharded matrix exactly
once with the unsharded model's bits. Launched by tests/test_tp_host.py under torchrun."""
import ctypes as C
import os
import sys

import numpy as np
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "vkllm.c_b200"))
import vkllm_b200 as vk  # noqa: E402

D, F, V = 64, 192, 96
KINDS = [("attn_q", D, D, 1), ("attn_output", D, D, 2), ("ffn_up", F, D, 1), ("ffn_down", D, F, 2),
         ("output", V, D, 1), ("token_embd", V, D, 0)]
SEED, STD = 5, 0.02


def main():
    dist.init_process_group("gloo", init_method="env://")
    rank, world = dist.get_rank(), dist.get_world_size()
    l = vk.lib()
    mine = []
    for tid, (name, rows, cols, split) in enumerate(KINDS):
        sp = (C.c_uint32 * 4)()
        assert l.vkllm_b200_tp_shard(rows, cols, split, rank, world, sp) == vk.OK
        r0, lr, c0, lc = list(sp)
        buf = np.zeros(lr * lc, dtype=np.uint16)
        l.vkllm_b200_random_f16_host_shard(SEED, tid, STD, cols, r0, lr, c0, lc, buf.ctypes.data)
        mine.append((name, r0, lr, c0, lc, buf.tobytes()))
    got = [None] * world
    dist.all_gather_object(got, mine)
    if rank == 0:
        for tid, (name, rows, cols, split) in enumerate(KINDS):
            full = np.zeros(rows * cols, dtype=np.uint16)
            l.vkllm_b200_random_f16_host(SEED, tid, STD, 0, rows * cols, full.ctypes.data)
            full = full.reshape(rows, cols)
            cover = np.zeros((rows, cols), dtype=np.int32)
            for q in range(world):
                n, r0, lr, c0, lc, b = got[q][tid]
                shard = np.frombuffer(b, dtype=np.uint16).reshape(lr, lc)
                assert (shard == full[r0:r0 + lr, c0:c0 + lc]).all(), (name, q)
                cover[r0:r0 + lr, c0:c0 + lc] += 1
            want = world if split == 0 else 1
            assert (cover == want).all(), (name, "coverage")
        # a shape that does not split evenly is refused
        sp = (C.c_uint32 * 4)()
        assert l.vkllm_b200_tp_shard(10, 8, 1, 0, 3, sp) == vk.ARGS
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
