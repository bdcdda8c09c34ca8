"""Pins the CPU oracle (oracle/) to golden vectors produced by the reference's own functions
(tests/golden/make_golden.py). CPU only."""
import hashlib

import numpy as np
import pytest

import vectors as V
from oracle import oracle as O


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_tables(golden):
    assert np.array_equal(O.e2m1_table().view(np.uint32), golden["e2m1"].view(np.uint32))
    t = O.e4m3_table()
    g = golden["e4m3"]
    nan = np.isnan(g)
    assert np.array_equal(np.isnan(t), nan)
    assert np.array_equal(t[~nan].view(np.uint32), g[~nan].view(np.uint32))


def test_deq_bit_exact_and_swap_control(golden):
    b = V.rand_block(1)
    w = b[V.O_UW:V.O_UW + 16 * 512].reshape(16, 512)
    s = b[V.O_US:V.O_US + 16 * 64].reshape(16, 64)
    assert np.array_equal(O.deq(w, s, 0.0123).view(np.uint32), golden["deq"].view(np.uint32))
    assert np.array_equal(O.deq(w, s, 0.0123, swap=True).view(np.uint32), golden["deq_swap"].view(np.uint32))
    # the swapped decode must differ (qmoe_ns.py:392 negative control)
    assert not np.array_equal(golden["deq"], golden["deq_swap"])


@pytest.mark.parametrize("seed", [2, 3])
def test_to_T_from_T_bit_exact(golden, seed):
    m = golden["meta"]
    blk = V.rand_bytes_block(seed)
    t = O.to_T(blk)
    assert sha(t) == m[f"to_T_{seed}"]
    assert sha(O.from_T(blk)) == m[f"from_T_{seed}"]
    assert np.array_equal(O.from_T(t), blk)          # tests/live_test.py:29-34 round trip
    assert np.array_equal(t[:V.O_DW], blk[:V.O_DW])  # up half untouched
    assert sha(O.from_T(t)) == m[f"from_T_batch_{seed}"]


def test_moe_decode_fp64(golden):
    blocks, s2, coef, x = V.decode_case()
    y, h, _ = O.moe_decode(blocks, s2, coef, x)
    gy, gh = golden["decode_y"], golden["decode_h"]
    assert np.abs(y - gy).max() <= 1e-10 * np.abs(gy).max()
    assert np.abs(h - gh).max() <= 1e-10 * np.abs(gh).max()
    # the T layout gives the same result (qmoe_ns.py:137-141: a pure byte permutation)
    bT = [O.to_T(b) for b in blocks]
    assert [sha(b) for b in bT] == golden["meta"]["decode_T_blocks_sha"]
    yT, hT, _ = O.moe_decode(bT, s2, coef, x, layoutT=True)
    assert np.abs(yT - gy).max() <= 1e-10 * np.abs(gy).max()


def test_live_groups_bit_exact(golden):
    gidx, gcnt = O.live_groups(golden["decode_h"].astype(np.float32))
    assert np.array_equal(gcnt, golden["decode_gcnt"])
    assert np.array_equal(gidx, golden["decode_gidx"])


def test_nibble_swap_control_diverges():
    """tests/kern_test.py:42-47: decoding with swapped nibbles must give a clearly different result."""
    blocks, s2, coef, x = V.decode_case()
    y, _, _ = O.moe_decode(blocks, s2, coef, x)
    u0 = O.deq(blocks[0][:V.O_US].reshape(2688, 512), blocks[0][V.O_US:V.O_DW].reshape(2688, 64), s2[0, 0])
    u1 = O.deq(blocks[0][:V.O_US].reshape(2688, 512), blocks[0][V.O_US:V.O_DW].reshape(2688, 64), s2[0, 0],
               swap=True)
    rel = np.linalg.norm(u0 @ x - u1 @ x) / np.linalg.norm(u0 @ x)
    assert rel > 0.1


def test_pairs_fp64(golden):
    blocks, pslot, ptok, s2p, coefp, X = V.pairs_case()
    out = O.pairs(blocks, pslot, ptok, s2p, coefp, X)
    g = golden["pairs_out"]
    assert np.abs(out - g).max() <= 1e-10 * np.abs(g).max()


@pytest.mark.parametrize("fmt,seed", [("fp8", 400), ("nvfp4", 401)])
def test_dense(golden, fmt, seed):
    w, sc, s, x = V.dense_case(fmt, seed)
    N = w.shape[0]
    K = w.shape[1] * (2 if fmt == "nvfp4" else 1)
    bits = O.dequant_rows_bf16(fmt, w, sc, s, K, 0, N)
    assert np.array_equal(bits, golden[f"dense_{fmt}_bf16"])
    y = O.dense(fmt, w, sc, s, N, K, x)
    g = golden[f"dense_{fmt}_y"]
    assert np.abs(y - g).max() <= 1e-10 * np.abs(g).max()


def test_cpu_fp32_path_matches_fp64():
    """The fp32 CPU baseline path (nem_super.py:342-346) agrees with the fp64 oracle."""
    blocks, s2, coef, x = V.decode_case()
    y64, _, _ = O.moe_decode(blocks, s2, coef, x)
    y32 = O.cpu_layer_fp32(blocks, s2, coef, x)
    assert np.linalg.norm(y32 - y64) / np.linalg.norm(y64) < 1e-5
    y32T = O.cpu_layer_fp32([O.to_T(b) for b in blocks], s2, coef, x, layoutT=True)
    assert np.linalg.norm(y32T - y64) / np.linalg.norm(y64) < 1e-5


def test_router_ids_match_transformers(golden):
    """tf:697-720 restated in qmoe_synth.route (n_group = topk_group = 1, top-22, x5.0) gives the same
    expert ids and weights as transformers' NemotronHMoE.route_tokens_to_experts on the golden inputs."""
    import torch
    import qmoe_synth as S
    h, w, b = V.route_case()
    ids, wt = S.route(torch.from_numpy(h), torch.from_numpy(w), torch.from_numpy(b))
    order = torch.argsort(ids, dim=1)
    assert np.array_equal(torch.gather(ids, 1, order).numpy(), golden["route_ids"])
    assert np.array_equal(torch.gather(wt, 1, order).numpy().view(np.uint32), golden["route_w"].view(np.uint32))
