"""Two gloo ranks on CPU: TP/EP shards reduce-scatter to the full-layer oracle output."""
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_sharding_matches_oracle():
    cmd = ["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           str(ROOT / "tests" / "dist_cpu_check.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert res.stdout.count("max rel err") == 4


def test_rank_that_never_joins_fails_fast():
    """A missing rank ends the others' rendezvous/collective with an error instead of a hang."""
    code = ("import datetime, torch.distributed as dist;"
            "dist.init_process_group('gloo', init_method='tcp://127.0.0.1:%d', rank=0, world_size=2,"
            " timeout=datetime.timedelta(seconds=3))" % _port())
    res = subprocess.run(["timeout", "-k", "5", "60", sys.executable, "-c", code], capture_output=True, text=True)
    assert res.returncode != 0
