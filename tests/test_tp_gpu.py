"""Tensor-parallel decode (BASELINE configs[4] layout: heads, FFN rows and vocabulary sharded) on 2
GPUs, with either exchange of the Wo / down partial sums: inside the persistent decode kernel over peer
memory ("peer"), or NCCL collectives between the per-op kernels ("nccl"), against the CPU oracle on
the unsharded weights (the generator is counter-based, so the oracle rebuilds them).
Each rank is a separate process (tests/multi/tp_decode_rank.py under torchrun). Bar: identical greedy
tokens on every rank and equal to the oracle's; the ranks' logit shards, concatenated, within
max-abs 2e-2 / mean-abs 2e-3 of the oracle's logits. Skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def oracle_weights(orc, cfg, seed):
    D, F, V, L = cfg["embedding_length"], cfg["ffn_length"], cfg["vocab_size"], cfg["block_count"]
    w, tid = {}, 0

    def mat(name, r, c):
        nonlocal tid
        w[name] = orc.random_f16(seed, tid, cfg["init_std"], 0, r * c).reshape(r, c)
        tid += 1

    def ones(name, n):
        nonlocal tid
        w[name] = np.ones(n, dtype=np.float32)
        tid += 1

    mat("token_embd.weight", V, D)
    for l in range(L):
        ones(f"blk.{l}.attn_norm.weight", D)
        ones(f"blk.{l}.ffn_norm.weight", D)
        for n in ("attn_q", "attn_k", "attn_v", "attn_output"):
            mat(f"blk.{l}.{n}.weight", D, D)
        mat(f"blk.{l}.ffn_gate.weight", F, D)
        mat(f"blk.{l}.ffn_up.weight", F, D)
        mat(f"blk.{l}.ffn_down.weight", D, F)
    ones("output_norm.weight", D)
    mat("output.weight", V, D)
    return w


@pytest.mark.parametrize("exchange,port", [("peer", 29533), ("nccl", 29534)])
def test_tensor_parallel_decode_matches_the_oracle(orc, tmp_path, exchange, port):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    sys.path.insert(0, os.path.join(HERE, "multi"))
    import tp_decode_rank as R

    env = dict(os.environ, MASTER_ADDR="127.0.0.1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={port}", os.path.join(HERE, "multi", "tp_decode_rank.py"), str(tmp_path), exchange]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    ranks = [np.load(os.path.join(tmp_path, f"rank{i}.npz")) for i in range(2)]
    toks = [list(map(int, x["toks"])) for x in ranks]
    assert toks[0] == toks[1]
    logits = np.concatenate([x["logits"] for x in ranks], axis=1)  # vocabulary shards in rank order

    cfg = R.CFG
    ocfg = dict(D=cfg["embedding_length"], H=cfg["head_count"], F=cfg["ffn_length"], V=cfg["vocab_size"],
                L=cfg["block_count"], ctx=cfg["context_length"], eps=cfg["rms_eps"], rope_base=cfg["rope_freq_base"])
    m = orc.Llama2(ocfg, oracle_weights(orc, cfg, R.SEED))
    ref_toks, ref_logits = [], []
    for i, t in enumerate(R.PROMPT):
        lg, am = m.step([t], i)
    ref_toks.append(int(am[-1]))
    ref_logits.append(lg[-1].copy())
    for g in range(R.N_GEN - 1):
        lg, am = m.step([ref_toks[-1]], len(R.PROMPT) + g)
        ref_toks.append(int(am[-1]))
        ref_logits.append(lg[-1].copy())
    m.close()
    assert toks[0] == ref_toks
    for s in range(R.N_GEN):
        d = np.abs(logits[s].astype(np.float32) - ref_logits[s].astype(np.float32))
        assert d.max() <= 2e-2 and d.mean() <= 2e-3, (s, d.max(), d.mean())
