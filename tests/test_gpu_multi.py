"""Multi-GPU parity of the NCCL and peer-memory schemes (skipped with fewer than 2 GPUs)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("scheme,preset,tokens,extra", [
    ("d1", "mixtral", 512, []), ("d3", "mixtral", 512, []),
    ("d2", "dsv3", 512, []), ("d4", "dsv3", 512, []), ("d4", "dsv3", 1024, ["--zipf"]),
    ("d3", "qwen3", 256, []),
    # copy-engine all-gather / reduce-scatter variants of the fused exchange
    ("d3", "mixtral", 512, ["--ag-mode", "ce", "--rs-mode", "ce", "--rs-chunks", "2"]),
    ("d4", "dsv3", 512, ["--ag-mode", "ce", "--rs-mode", "ce", "--rs-chunks", "1"]),
    ("d3", "mixtral", 512, ["--ag-mode", "ce"]),
    # down GEMM storing straight into the owners' receive buffers
    ("d3", "mixtral", 512, ["--rs-mode", "gemm"]),
    ("d4", "dsv3", 1024, ["--zipf", "--rs-mode", "gemm"]),
    ("d3", "qwen3", 256, ["--rs-mode", "gemm"]),
    # all-gather stored straight into the peers' sorted operand under the gate/up GEMM
    ("d3", "mixtral", 512, ["--ag-mode", "push"]),
    ("d3", "mixtral", 1024, ["--ag-mode", "push", "--rs-mode", "gemm"]),
    ("d3", "qwen3", 256, ["--ag-mode", "push"]),
    # FP8 reduce-scatter payload (the b3 variant): peer memory and NCCL all-to-all
    ("d3", "mixtral", 512, ["--rs-dtype", "fp8"]),
    ("d4", "dsv3", 1024, ["--zipf", "--rs-dtype", "fp8"]),
    ("d1", "mixtral", 512, ["--rs-dtype", "fp8"]),
    ("d2", "dsv3", 512, ["--rs-dtype", "fp8"]),
    # sparse expert-parallel exchange (bit-identical to the dense one)
    ("d4", "dsv3", 1024, ["--zipf", "--sparse"]),
    ("d4", "dsv3", 512, ["--sparse", "--rs-dtype", "fp8"]),
    ("d4", "dsv3", 1024, ["--zipf", "--sparse", "--rs-mode", "gemm"]),
    # experts placed by routed load instead of contiguous ranges (same output within the gates)
    ("d4", "dsv3", 1024, ["--zipf", "--placement", "balanced"]),
    ("d4", "dsv3", 1024, ["--zipf", "--placement", "balanced", "--sparse", "--rs-dtype", "fp8"]),
    ("d2", "dsv3", 512, ["--zipf", "--placement", "balanced"]),
], ids=lambda v: "-".join(a.strip("-") for a in v) if isinstance(v, list) else str(v))
def test_multi_gpu_scheme_matches_golden(scheme, preset, tokens, extra):
    n = min(_gpus(), 4)
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           str(ROOT / "tests" / "dist_gpu_check.py"), "--scheme", scheme, "--preset", preset, "--tokens", str(tokens),
           *extra]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, env=env)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert '"pass": true' in res.stdout
