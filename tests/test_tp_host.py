"""CPU, world size 2 (gloo): the tensor-parallel weight layout. Each rank's shards (from the
library's shard geometry and the host twin of the device generator) must tile every unsharded
matrix exactly once with the unsharded model's bits; see tests/multi/tp_shard_rank.py."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def test_tp_shards_tile_the_unsharded_matrices_world_2():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           "--master-port=29541", os.path.join(HERE, "multi", "tp_shard_rank.py")]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
