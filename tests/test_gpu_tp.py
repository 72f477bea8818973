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


def _run(tmp_path: Path, ranks: int, kv_heads: int, heads: int = 4, head_dim: int = 64, extra: tuple = ()) -> None:
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={ranks}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(ROOT / "tests" / "tp_worker.py"),
           "--out", str(out), "--kv-heads", str(kv_heads), "--heads", str(heads), "--head-dim", str(head_dim),
           *extra]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600, check=False)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["ok"], res


@pytest.mark.parametrize("kv_heads", [1, 2])
def test_tensor_parallel_decode_matches_oracle(tmp_path: Path, kv_heads: int) -> None:
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    _run(tmp_path, 2, kv_heads)


@pytest.mark.parametrize("ranks", [4, 8])
def test_tensor_parallel_27b_head_geometry(tmp_path: Path, ranks: int) -> None:
    """Gemma3-27B's head geometry (head dim 128, 2 q heads per kv head: 16 q / 8 kv heads here) split over 4
    and 8 ranks: every rank keeps 2 or 1 kv heads with their q heads."""
    if _gpus() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    _run(tmp_path, ranks, kv_heads=8, heads=16, head_dim=128)


def test_tensor_parallel_split_row_groups(tmp_path: Path) -> None:
    """bf16 hidden 2560, FFN 8192 over 2 ranks: each rank's down_proj has 160 row groups of 4 tiles for 148
    CTAs, so its tiles are split evenly and the CTAs that share a group add their partial sums before the rows
    go to every rank's exchange buffer."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    _run(tmp_path, 2, kv_heads=2, heads=4, head_dim=256,
         extra=("--hidden", "2560", "--intermediate", "8192", "--bf16"))
