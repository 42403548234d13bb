"""Multi-GPU paths on real GPUs (skipped with fewer than two): head-sharded causal prefill
(all-gather by NCCL, and fused into the attention kernel's epilogue over NVLink) and
value-head-sharded chunked DeltaNet prefill over 2 ranks (torchrun, NCCL) against the
unsharded call on one GPU — identical per-head arithmetic, so identical outputs and state."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_head_sharded_prefill_two_ranks(tmp_path):
    out = tmp_path / "sharded.npz"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "mgpu_prefill_worker.py"), str(out)]
    r = subprocess.run(["timeout", "-k", "30", "240"] + cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    d = np.load(out)
    assert int(d["world"]) == 2
    np.testing.assert_array_equal(d["sharded"], d["full"])
    # the all-gather fused into the attention kernel: every rank's copy equals the unsharded output
    assert int(d["fused_ok_ranks"]) == 2
    np.testing.assert_array_equal(d["fused"], d["full16"])


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_value_head_sharded_deltanet_two_ranks(tmp_path):
    out = tmp_path / "sharded_gdn.npz"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "mgpu_gdn_worker.py"), str(out)]
    r = subprocess.run(["timeout", "-k", "30", "240"] + cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    d = np.load(out)
    assert int(d["world"]) == 2
    np.testing.assert_array_equal(d["sharded"], d["full"])
    np.testing.assert_array_equal(d["state_sharded"], d["state_full"])
