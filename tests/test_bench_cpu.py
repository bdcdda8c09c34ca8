"""bench.py on the CPU: the reference arms' JSON lines (decode and prefill) carry the contract's keys, the
prefill reference arm computes the reference's prompt path (per-expert block_deq + two fp32 linears,
nem_super.py:342-346) and agrees with the fp64 oracle, and the clock sampler degrades to a marked
"unavailable" record without a GPU."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "nemotron-super-8gb_b200"))

import bench  # noqa: E402
import qmoe_synth as S  # noqa: E402
from oracle import oracle as O  # noqa: E402

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _run(*argv, env=None):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *argv], capture_output=True, text=True,
                       timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_prefill_reference_arm_line():
    line = json.loads(_run("--impl", "reference", "--workload", "prefill", "--prefill-t", "64", "--steps", "1",
                           "--warmup", "0").strip().splitlines()[-1])
    assert KEYS <= set(line)
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["metric"] == bench.PREFILL_METRIC and line["config"]["T"] == 64 and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    assert _run("--impl", "reference", "--workload", "prefill", "--prefill-t", "64", "--steps", "1",
                "--warmup", "0", env=env).strip() == ""


def test_prefill_cpu_reference_matches_oracle():
    g = S.seeded(7, "cpu")
    m_hat = S.unit_dir(g, "cpu")
    E, T, k = 6, 24, 3
    blk, s2, _ = S.expert_blocks(E, 0.1, m_hat, g, "cpu")
    blocks = blk.numpy()
    s2 = s2.numpy()
    X = S.tokens(T, m_hat, g, "cpu").float().numpy()
    rng = np.random.default_rng(0)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    ids[3, 1] = -1                                   # a "no expert" slot is skipped
    w = rng.random((T, k)).astype(np.float32)
    v, n, sample, out = bench.prefill_cpu_reference(lambda e: blocks[e], s2, ids, w, X, threads=2,
                                                    max_experts=E, return_out=True)
    assert v > 0 and n == 2 and f"of the {E} experts" in sample
    ref = O.prefill(list(blocks), s2, ids, w, X)
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel < 1e-5


def test_clock_sampler_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    c = bench.Clocks(0)
    c.start()
    rec = c.stop()
    assert rec["sm_mhz"] is None or rec["sm_mhz"] > 0
    assert "reasons" in rec


def test_dense_cpu_reference():
    g = S.seeded(9, "cpu")
    qs = []
    for fmt, N, K in (("fp8", 64, 128), ("nvfp4", 48, 256)):
        wf = torch.randn(N, K, generator=g) * 0.02
        if fmt == "fp8":
            codes, s_ = S.quantize_fp8(wf)
            q = {"fmt": "fp8", "w": codes.numpy(), "s": s_.reshape(1).numpy(), "N": N, "K": K}
        else:
            codes, sc, s2 = S.quantize_nvfp4(wf)
            q = {"fmt": "nvfp4", "w": codes.numpy(), "sc": sc.numpy(), "s": s2.reshape(1).numpy(), "N": N, "K": K}
        qs.append((q, torch.randn(K, generator=g).numpy()))
    us = bench.dense_cpu_reference(qs)
    assert len(us) == 2 and all(u is not None and u > 0 for u in us)
    assert bench.dense_cpu_reference(qs, budget_s=-1.0) == [None, None]   # past the budget: skipped


def test_dense_and_ep_reference_arms():
    line = json.loads(_run("--impl", "reference", "--workload", "dense", "--steps", "1", "--warmup", "0")
                      .strip().splitlines()[-1])
    assert KEYS <= set(line)
    assert line["metric"] == bench.DENSE_METRIC and line["higher_is_better"] is False and line["value"] > 0
    ep = json.loads(_run("--impl", "reference", "--workload", "ep", "--steps", "1", "--warmup", "0").strip())
    assert ep["impl"] == "reference" and "unavailable" in ep


def test_decode_reference_path_matches_oracle(monkeypatch):
    """The decode reference arm's code (decode_token_inputs + decode_cpu_token: the reference's fp32 CPU expert
    path per layer) on a tiny store: both layouts give the same host blocks, and each layer's fp32 result is
    within 1e-5 of the fp64 oracle."""
    monkeypatch.setattr(bench, "NE", 4)
    g = S.seeded(3, "cpu")
    m_hat = S.unit_dir(g, "cpu")
    L, k = 2, 3
    blk, s2, _ = S.expert_blocks(L * 4, 0.1, m_hat, g, "cpu")
    storeT = torch.from_numpy(np.stack([O.to_T(b) for b in blk.numpy()]))
    T = {"IDS": torch.tensor([[[0, 2, 3], [1, 2, 0]]]), "W": torch.rand(1, L, k, generator=g),
         "X": S.tokens(L, m_hat, g, "cpu").view(1, L, 1024)}
    s2h = s2.view(L, 4, 2).numpy()
    layers = bench.decode_token_inputs(blk, s2h, T, 0, L, layout_T=False)
    layersT = bench.decode_token_inputs(storeT, s2h, T, 0, L, layout_T=True)
    for (b0, *_), (b1, *_) in zip(layers, layersT):
        assert all(np.array_equal(a, b) for a, b in zip(b0, b1))
    assert bench.decode_cpu_token(layers, 2) > 0
    for blocks, s2m, coef, x in layers:
        y32 = O.cpu_layer_fp32(blocks, s2m, coef, x, nthreads=2)
        y64, _, _ = O.moe_decode(blocks, s2m, coef, x)
        assert np.linalg.norm(y32 - y64) / np.linalg.norm(y64) < 1e-5
    assert bench.decode_config(40, 1) == bench.decode_config(40, 1) and "parallelism" in bench.decode_config(40, 2)
