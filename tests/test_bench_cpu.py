"""CPU checks of bench.py's CPU legs: the reference arm and the `cpu_baseline` object
run without a GPU and without this repository's kernels, and the timed CPU port
computes the reference pipeline's result."""
import json
import os
import subprocess
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpu_reference_run_small_sample():
    sys.path.insert(0, ROOT)
    import bench
    r = bench.cpu_reference_run(64, steps=1, warmup=1, threads=2, budget_s=1.0)
    assert r["value"] > 0 and r["kind"] == "port" and r["cores"] == 2
    assert 1 <= r["experts_per_sample"] <= bench.E


def test_cpu_baseline_reports_errors_instead_of_raising(monkeypatch):
    sys.path.insert(0, ROOT)
    import bench

    def boom(*a, **k):
        raise RuntimeError("planted")
    monkeypatch.setattr(bench, "cpu_reference_run", boom)
    r = bench.cpu_baseline(64, threads=1)
    assert r["value"] is None and "planted" in r["error"]


def test_reference_arm_prints_one_line_without_repo_kernels():
    code = ("import sys, runpy; sys.argv = ['bench.py', '--impl', 'reference', '--M', '32', '--steps', '1', "
            "'--warmup', '1']; runpy.run_path('bench.py', run_name='__main__'); "
            "assert 'aiter_b200' not in sys.modules, 'reference arm imported aiter_b200'")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, env=env,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    res = json.loads(lines[0])
    assert res["impl"] == "reference" and res["value"] > 0
    assert res["e2e"]["h2d_bytes_per_step"] == 0 and res["cpu_baseline"]["kind"] == "port"


def test_reference_arm_other_ranks_exit_without_work():
    code = ("import sys, runpy; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '1']; "
            "runpy.run_path('bench.py', run_name='__main__')")
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, env=env,
                         timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == ""


def test_threaded_numpy_port_equals_serial_oracle():
    sys.path.insert(0, ROOT)
    from oracle import inputs, moe
    c = inputs.make_moe_case(0, 32, 1024, 512, 8, 2)
    a = moe.fused_moe_fp8_blockscale_threaded(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                              c["topk_weights"], c["topk_ids"], threads=2)
    b = moe.fused_moe_fp8_blockscale(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                     c["topk_weights"], c["topk_ids"])
    assert np.array_equal(a, b)


def test_torch_port_expert_sample_covers_the_full_result():
    """Processing the experts in disjoint samples and adding the per-sample outputs
    (before the final bf16 rounding the sums differ) touches every routed row once:
    the union of samples with all experts equals the one-call result."""
    sys.path.insert(0, ROOT)
    from oracle import inputs, moe_torch as mt
    c = inputs.make_moe_case(3, 16, 256, 128, 8, 2)
    fp8 = lambda a: torch.from_numpy(a).view(torch.float8_e4m3fn)
    args = (torch.from_numpy(c["hidden"]).to(torch.bfloat16), fp8(c["w1_q"]), torch.from_numpy(c["w1_s"]),
            fp8(c["w2_q"]), torch.from_numpy(c["w2_s"]), torch.from_numpy(c["topk_weights"]),
            torch.from_numpy(c["topk_ids"]))
    full = mt.fused_moe_fp8_blockscale(*args)
    tm = {}
    same = mt.fused_moe_fp8_blockscale(*args, experts=list(range(8)), timer=tm)
    assert torch.equal(full, same) and tm["experts"] > 0 and tm["shared"] > 0
