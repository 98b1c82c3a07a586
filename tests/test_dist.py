"""The benchmark's N-process path (one process per GPU, replicas, no
collective on the data path) on host cores: torchrun with the gloo backend,
world size 2.  The ranks meet at barriers and agree on the slowest rank's
time and the job's token total, which make the whole-job throughput."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_aggregate_over_gloo(tmp_path):
    env = dict(os.environ, JL_DIST_BACKEND="gloo", OMP_NUM_THREADS="1", JL_DIST_OUT=str(tmp_path))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", str(HERE / "dist_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [json.loads(p.read_text()) for p in sorted(tmp_path.glob("rank*.json"))]
    assert sorted(x["rank"] for x in lines) == [0, 1]
    for x in lines:
        assert x["world"] == 2
        assert x["tokens"] == 64 + 65
        # every rank's tokens over the slowest rank's time (200 ms device, 2 s wall)
        assert abs(x["value"] - 129 / 0.2) < 1e-9
        assert abs(x["e2e"] - 129 / 2.0) < 1e-9
        assert x["slowest_ms"] == 200.0


def test_every_benchmark_model_is_placed_on_the_ranks_gpu():
    """Under torchrun each rank builds its models on its own GPU
    (LOCAL_RANK): a model left on GPU 0 fails a speculative call with a draft
    on the rank's GPU.  Every model the benchmark synthesises passes a device."""
    import re

    src = (HERE.parent / "bench.py").read_text()

    def call_args(pattern):
        out = []
        for m in re.finditer(pattern, src):
            depth, i = 0, src.index("(", m.start())
            for j in range(i, len(src)):
                depth += {"(": 1, ")": -1}.get(src[j], 0)
                if depth == 0:
                    break
            out.append(src[i:j + 1])
        return out

    calls = call_args(r"Model\.synthesize\(")
    assert calls
    for args in calls:
        assert "device=" in args or "**opts" in args, args
    for args in call_args(r"opts = dict\("):
        assert "device=" in args, args
