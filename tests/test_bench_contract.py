"""bench.py's output contract, checked on CPU through its reference arm (the CPU oracle timed on the
host cores, which needs no GPU): one JSON line with the metric, the timing fields, the CPU-baseline
description and an e2e entry with no host/device copies; under torchrun only rank 0 prints it and
every rank exits 0.  Our arm, with no GPU visible, exits non-zero without printing a line."""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CONFIGS = ["gdn_decode", "gdn_prefill", "kv_attention", "gdn_layer", "cache_ops"]


def _run(args, timeout=300):
    r = subprocess.run(args, cwd=ROOT, capture_output=True, text=True, timeout=timeout,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]


def _check_line(d, config):
    assert d["impl"] == "reference"
    for k in ("metric", "unit", "ms_per_step", "higher_is_better", "scaling", "dtype", "data", "config"):
        assert k in d, k
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["steps"] == 1 and d["warmup"] >= 3  # the contract's minimum of three warm-up steps
    assert d["vs_baseline"] is None
    assert d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    sys.path.insert(0, ROOT)
    import bench
    # the config dict is the one our arm prints for the same workload
    assert d["config"] == bench.reference_config(config or "gdn_decode", d["n_gpus"], 0)
    if config is None:  # the default run carries the prefill and KV attention lines too
        for key, cfg, window in bench.SECONDARY:
            sub = d[key]
            assert sub["metric"] == bench.METRICS[cfg] and sub["value"] > 0 and sub["unit"] == "tokens/s"
            assert sub["config"] == bench.reference_config(cfg, d["n_gpus"], window)
            assert sub["cpu_baseline"]["value"] == sub["value"]


@pytest.mark.parametrize("config", CONFIGS + [None])
def test_reference_arm_prints_one_contract_line(config):
    cfg_args = [] if config is None else ["--config", config]
    lines = _run([sys.executable, "bench.py", "--impl", "reference", *cfg_args, "--steps", "1", "--warmup", "1"])
    assert len(lines) == 1
    _check_line(lines[0], config)


def test_reference_arm_under_torchrun_prints_once():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    lines = _run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                  "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                  "--config", "cache_ops", "--steps", "1", "--warmup", "1"])
    assert len(lines) == 1
    _check_line(lines[0], "cache_ops")


@pytest.mark.parametrize("config", ["gdn_decode", "stack"])
def test_our_arm_fails_loudly_without_a_gpu(config):
    """The library path has no CPU fallback: without a GPU our arm exits non-zero and prints no line."""
    r = subprocess.run([sys.executable, "bench.py", "--config", config, "--steps", "1"], cwd=ROOT,
                       capture_output=True, text=True, timeout=300, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode != 0
    assert not any(l.startswith("{") for l in r.stdout.splitlines())
