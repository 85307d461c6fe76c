"""Tensor parallelism on 2, 4 and 8 GPUs: the sharded model (column-split q/k/v, gate/up; row-split
o, down with an int32 all-reduce; vocab-split LM head) against the one-GPU oracle, bit
for bit.  Each case needs that many visible GPUs; skipped otherwise."""
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_bit_exact_against_oracle(tmp_path, world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    # the workers abort on a peer's failure within a second and give up after 180 s;
    # the outer timeout is the last bound
    cmd = ["timeout", "-k", "60", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "tp_worker.py"), str(tmp_path / "failed")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
