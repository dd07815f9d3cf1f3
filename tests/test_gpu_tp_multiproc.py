"""Tensor parallelism with one process per GPU (needs >= 2 GPUs; skipped otherwise):
the NCCL path and the fused NVLink allreduce path (inside a CUDA graph) agree, and
every rank ends with the same tokens and slot tables.  The ranks run as child processes
under torchrun with a short process-group timeout and an outer time limit."""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from kvcacheboundaryprotection_b200 import build

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_fused_allreduce_matches_nccl(tmp_path):
    build.build()
    out = tmp_path / "tp2.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), os.path.join(HERE, "mp_tp_worker.py"), str(out)]
    r = subprocess.run(cmd, timeout=600, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["tokens_equal_across_ranks"] and res["slot_tables_equal"]
    assert res["max_logit_diff"] <= 2e-2, res["max_logit_diff"]
    assert res["argmax_decisive"] >= 10 and res["argmax_agree"] >= 0.99 * res["argmax_decisive"]
    assert res["evlog_a"] == res["evlog_b"]
