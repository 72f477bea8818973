"""Tensor-parallel decode (2 GPUs) against the oracle and the single-GPU engine.

Each case launches tests/tp_worker.py on two ranks (one process per GPU,
torch.distributed over NCCL for the handle exchange; the o_proj / down_proj
partial sums and the lm_head candidates cross NVLink inside the decode kernel).
Checked: gathered logits within the logits tolerance of the oracle, identical
greedy and top-k streams on every rank, and greedy tokens equal to one GPU's.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _gpus() -> int:
    try:
        import torch  # noqa: PLC0415

        return torch.cuda.device_count()
    except Exception:  # noqa: BLE001
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


@pytest.mark.parametrize("kv_heads", [1, 2])
def test_tensor_parallel_decode_matches_oracle(tmp_path: Path, kv_heads: int) -> None:
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(ROOT / "tests" / "tp_worker.py"),
           "--out", str(out), "--kv-heads", str(kv_heads)]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600, check=False)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["ok"], res
