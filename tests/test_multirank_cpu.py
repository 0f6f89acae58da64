"""The N > 1 host logic of bench.py on CPU: two gloo ranks shard the job's sequences without a
data-path collective and take the max of their timings; the reference arm launched under
torchrun prints one line, from rank 0, for the whole job."""
import json
import os
import socket
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        res = {}
        for name in ("cfg1", "cfg2", "cfg4"):
            per, job = bench.rank_batch(bench.CONFIGS[name], world)
            rows = list(range(job))[bench.rank_rows(rank, per)]
            res[name] = (per, job, rows)
        res["max"] = bench.max_over_ranks(10.0 + rank, world, torch.device("cpu"))
        out[rank] = res
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_sequences_and_take_the_max_time():
    world, port = 2, _free_port()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
    for name, (per_exp, job_exp) in {"cfg1": (1, 2), "cfg2": (32, 64), "cfg4": (128, 256)}.items():
        rows = []
        for r in range(world):
            per, job, rws = out[r][name]
            assert (per, job) == (per_exp, job_exp)
            rows += rws
        assert rows == list(range(job_exp))  # disjoint, contiguous, complete
    assert out[0]["max"] == out[1]["max"] == 11.0


def test_reference_arm_under_torchrun_prints_one_job_line():
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"),
           "--impl", "reference", "--config", "cfg0", "--gpus", "2", "--steps", "2", "--warmup", "3"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference"
    if "unavailable" not in line:
        assert line["config"]["global_batch"] == 2 and line["n_gpus"] == 2 and line["value"] > 0
        # the same workload keys and values as the engine's arm prints for cfg0 at two ranks
        from dfssm_b200 import synthetic
        cfg = bench.CONFIGS["cfg0"]
        d = synthetic.make_dims(cfg["shape"], cfg["layers"])
        assert line["config"] == bench.workload_config("cfg0", cfg, 1, 2, bench.step_bytes(d, 1)["total"])


@pytest.mark.parametrize("config", ["cfg3", "cfg1 --prefill 16"])
def test_reference_arm_without_a_counterpart_prints_unavailable(config):
    """The reference has no stand-alone scaffold GEMM entry point and no prompt prefill, so the
    reference arm of those workloads prints one 'unavailable' line and exits 0 (no GPU needed)."""
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", *config.split()]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["unavailable"]


def test_roofline_bytes_per_step():
    """Algorithmic HBM bytes of one decode step, the numerator of bench.py's roofline: packed
    scaffold, fp16 scales, int8 LoRA, conv/SSM parameters and norms (173.1 MB at 48 layers of the
    1.3B shape), the int8 embedding with its scales (103.2 MB) and per sequence the fp32 SSM and
    conv state read and written (206.3 MB)."""
    from dfssm_b200 import synthetic
    d = synthetic.make_dims("1.3b", 48)
    one, many = bench.step_bytes(d, 1), bench.step_bytes(d, 32)
    assert (one["weights"], one["embedding"], one["state"]) == (173100032, 103174560, 206340096)
    assert one["total"] == 482614688
    assert many["state"] == 32 * one["state"] and many["total"] == one["total"] + 31 * one["state"]
