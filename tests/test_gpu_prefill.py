"""GPU parity of the prompt path qmoe_prefill_grouped (tcgen05 expert-grouped GEMM) through the drop-in
qmoe_ns.moe_prefill, against the fp64 oracle of moe_pairs (qmoe_ns.py:79-133) combined over top-k in k
order (nem_super.py:309-347), and against the reference's own moe_pairs golden vector.

Bars: rel-L2 <= 2^-8 (BF16_TOL) of the fp64 oracle for every token (the activations enter the block-scaled
NVFP4 MMA as three NVFP4 residual planes, ~8e-4; h is stored as f32); deterministic bit-identical reruns;
the T and orig layouts give identical results; an invalid expert id is reported and poisons only its own token.
"""
import numpy as np
import pytest
import torch

import vectors as V
from oracle import oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 2.0 ** -8
DEV = "cuda"


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def Q():
    import qmoe_ns
    return qmoe_ns


def oracle_prefill(blocks_np, s2_np, ids, w, X):
    """fp64 pairs oracle + fixed-order combine over k."""
    T, k = ids.shape
    pslot = ids.reshape(-1).astype(np.int32)
    ptok = np.repeat(np.arange(T, dtype=np.int32), k)
    out = O.pairs(list(blocks_np), pslot, ptok, s2_np[pslot], w.reshape(-1).astype(np.float32), X)
    return out.reshape(T, k, -1).sum(1)


@pytest.fixture(scope="module")
def bank():
    """24 synthetic experts (config 0 recipe), orig and T layouts, and 48 tokens."""
    import qmoe_synth as S
    g = S.seeded(23, DEV)
    m_hat = S.unit_dir(g, DEV)
    blk, s2, _ = S.expert_blocks(24, 0.075, m_hat, g, DEV)
    X = S.tokens(48, m_hat, g, DEV)
    blkT = blk.clone()
    import qmoe_ns
    qmoe_ns.to_T_batch(blkT)
    torch.cuda.synchronize()
    return dict(blk=blk, blkT=blkT, s2=s2.float().contiguous(), X=X, blk_np=blk.cpu().numpy(),
                s2_np=s2.float().cpu().numpy(), X_np=X.float().cpu().numpy())


def _route(T, E, k, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, (T, k)).astype(np.float32)
    return ids, w


def test_prefill_golden_pairs(Q, golden):
    """The reference's moe_pairs golden output (random-byte blocks), combined over k, both layouts."""
    blocks, pslot, ptok, s2p, coefp, X = V.pairs_case()
    T = int(ptok.max()) + 1
    k = len(pslot) // T
    ids = pslot.reshape(T, k)
    w = coefp.reshape(T, k)
    rng = np.random.default_rng(200)          # s2 per block, as pairs_case draws it
    s2 = rng.uniform(0.002, 0.02, (len(blocks), 2)).astype(np.float32)
    assert np.array_equal(s2[pslot], s2p)
    ref = golden["pairs_out"].reshape(T, k, -1).sum(1)
    store = torch.from_numpy(np.stack(blocks)).to(DEV)
    Xd = torch.from_numpy(X).to(DEV).to(torch.bfloat16)
    y = Q.moe_prefill(store, torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV),
                      torch.from_numpy(s2).to(DEV), Xd, layout_T=False)
    assert Q.prefill_status() == 0
    assert rel_l2(y.cpu().numpy(), ref) < BF16_TOL
    storeT = store.clone()
    Q.to_T_batch(storeT)
    yT = Q.moe_prefill(storeT, torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV),
                       torch.from_numpy(s2).to(DEV), Xd, layout_T=True)
    # a T-layout store has its used down halves converted to the orig layout first: the same GEMMs, bit for bit
    assert rel_l2(yT.cpu().numpy(), ref) < BF16_TOL
    assert torch.equal(yT, y)


@pytest.mark.parametrize("T,k", [(1, 1), (1, 22), (37, 8), (48, 22)])
def test_prefill_vs_oracle(Q, bank, T, k):
    b = bank
    ids, w = _route(T, 24, k, seed=T * 100 + k)
    ref = oracle_prefill(b["blk_np"], b["s2_np"], ids, w, b["X_np"][:T])
    for layout_T, store in ((True, b["blkT"]), (False, b["blk"])):
        y = Q.moe_prefill(store, torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV), b["s2"], b["X"][:T],
                          layout_T=layout_T)
        assert Q.prefill_status() == 0
        yn = y.cpu().numpy()
        assert np.isfinite(yn).all()
        assert rel_l2(yn, ref) < BF16_TOL
        for t in range(T):
            assert rel_l2(yn[t], ref[t]) < BF16_TOL


def test_prefill_multi_tile_experts(Q, bank):
    """Experts with more than 256 pairs are split into several tiles (N = 256 + remainder)."""
    b = bank
    T, E, k = 300, 2, 2
    Xs = b["X"].repeat(7, 1)[:T] + 0
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    Xs = (Xs.float() + 0.05 * torch.randn(Xs.shape, generator=g, device=DEV)).to(torch.bfloat16)
    ids, w = _route(T, E, k, seed=77)
    assert np.bincount(ids.ravel(), minlength=E).min() > 256   # 2 tiles per expert
    ref = oracle_prefill(b["blk_np"][:E], b["s2_np"][:E], ids, w, Xs.float().cpu().numpy())
    y = Q.moe_prefill(b["blkT"][:E], torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV), b["s2"][:E], Xs)
    assert Q.prefill_status() == 0
    yn = y.cpu().numpy()
    assert rel_l2(yn, ref) < BF16_TOL
    assert max(rel_l2(yn[t], ref[t]) for t in range(T)) < BF16_TOL


def test_prefill_deterministic_and_matches_decode(Q, bank):
    b = bank
    T, k = 24, 22
    ids, w = _route(T, 24, k, seed=9)
    idd, wd = torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV)
    y1 = Q.moe_prefill(b["blkT"], idd, wd, b["s2"], b["X"][:T])
    y2 = Q.moe_prefill(b["blkT"], idd, wd, b["s2"], b["X"][:T])
    assert torch.equal(y1, y2)
    # the decode path (W4A16 GEMV kernels) agrees per token
    for t in (0, 13):
        sel = idd[t].int().contiguous()
        tab = torch.tensor([b["blkT"][int(j)].data_ptr() for j in ids[t]], dtype=torch.int64, device=DEV)
        yd = Q.moe_decode_groups(b["blkT"], sel, tab, b["s2"][sel.long()].contiguous(), wd[t].contiguous(),
                                 b["X"][t], torch.empty(k, 2688, device=DEV), torch.empty(2, k, 1024, device=DEV),
                                 torch.empty(k, 168, dtype=torch.int32, device=DEV),
                                 torch.empty(k, dtype=torch.int32, device=DEV))
        assert rel_l2(y1[t].cpu().numpy(), yd.cpu().numpy()) < BF16_TOL


def test_prefill_invalid_id_poisons_only_its_token(Q, bank):
    b = bank
    T, k = 6, 4
    ids, w = _route(T, 24, k, seed=3)
    bad = ids.copy()
    bad[2, 1] = 24          # out of range
    y = Q.moe_prefill(b["blkT"], torch.from_numpy(bad).to(DEV), torch.from_numpy(w).to(DEV), b["s2"], b["X"][:T])
    assert Q.prefill_status() == 1        # QMOE_ERR_SHAPE recorded on the device
    assert Q.prefill_status() == 0        # and cleared
    yn = y.cpu().numpy()
    assert np.isnan(yn[2]).all()
    good = [t for t in range(T) if t != 2]
    ref = oracle_prefill(b["blk_np"], b["s2_np"], ids[good], w[good], b["X_np"][good])
    assert rel_l2(yn[good], ref) < BF16_TOL


def test_prefill_T_layout_in_cuda_graph(Q, bank):
    """The T-layout call forks its down-half conversion onto a side stream and joins it back: recorded in a
    CUDA graph and replayed, it gives the eager result."""
    b = bank
    T, k = 24, 8
    ids, w = _route(T, 24, k, seed=41)
    idd, wd = torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV)
    X = b["X"][:T].clone()
    y_eager = Q.moe_prefill(b["blkT"], idd, wd, b["s2"], X, layout_T=True).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        Q.moe_prefill(b["blkT"], idd, wd, b["s2"], X, layout_T=True)   # this stream's workspace, before capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        y_graph = Q.moe_prefill(b["blkT"], idd, wd, b["s2"], X, layout_T=True)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_graph, y_eager)
    del g


def test_prefill_wait_limit_times_out_and_recovers(Q, bank):
    """qmoe_set_wait_cycles(300): a wait of the GEMM pipeline runs out long before its copies land, the call
    records QMOE_ERR_TIMEOUT (4) in the workspace status, and the kernels stop after every copy and MMA in
    flight has completed. With the default bound restored, the next call is clean and bit-identical to a
    call made before the timeout (the context and the workspace stay usable)."""
    b = bank
    T, k = 48, 22
    ids, w = _route(T, 24, k, seed=77)
    idd, wd = torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV)
    y_ref = Q.moe_prefill(b["blkT"], idd, wd, b["s2"], b["X"][:T]).clone()
    assert Q.prefill_status() == 0
    seen = []
    Q.set_wait_cycles(300)
    try:
        for _ in range(3):
            Q.moe_prefill(b["blkT"], idd, wd, b["s2"], b["X"][:T])
            seen.append(Q.prefill_status())
            if seen[-1] == 4:
                break
    finally:
        Q.set_wait_cycles(0)
    assert seen[-1] == 4 and set(seen) <= {0, 4}, seen
    y = Q.moe_prefill(b["blkT"], idd, wd, b["s2"], b["X"][:T])
    assert Q.prefill_status() == 0
    assert torch.equal(y, y_ref)


def test_prefill_every_box_height(Q, bank):
    """Tiles of 1, 15, 16, 17, 31, 32, 33, 40, 47, 48, 49, 63, 64, 65, 79, 80, 81, 95, 96, 97, 111, 112, 113, 127
    and 128 pairs (one expert each, k = 1): every plane box height (16, 32, then 48 ... 128 rows), every MMA
    width, the fused-plane and the per-plane MMAs, in both layouts, each token against the fp64 oracle."""
    b = bank
    sizes = [1, 15, 16, 17, 31, 32, 33, 40, 47, 48, 49, 63, 64, 65, 79, 80, 81, 95, 96, 97, 111, 112, 113, 127]
    sizes = sizes + [128]                       # the 25th size goes to expert 0 again: a second tile of it
    experts = [i % 24 for i in range(len(sizes))]
    ids = np.concatenate([np.full(n, e, dtype=np.int32) for n, e in zip(sizes, experts)])[:, None]
    T = ids.shape[0]
    rng = np.random.default_rng(11)
    perm = rng.permutation(T)                   # tokens of one expert spread over the prompt
    ids = ids[perm]
    w = rng.uniform(0.1, 1.0, (T, 1)).astype(np.float32)
    g = torch.Generator(device=DEV)
    g.manual_seed(9)
    X = (b["X"].repeat(T // 48 + 1, 1)[:T].float() * (1 + 0.1 * torch.rand(T, 1, generator=g, device=DEV))).to(torch.bfloat16)
    ref = oracle_prefill(b["blk_np"], b["s2_np"], ids, w, X.float().cpu().numpy())
    outs = []
    for layout_T, store in ((True, b["blkT"]), (False, b["blk"])):
        y = Q.moe_prefill(store, torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV), b["s2"], X,
                          layout_T=layout_T)
        assert Q.prefill_status() == 0
        yn = y.cpu().numpy()
        assert max(rel_l2(yn[t], ref[t]) for t in range(T)) < BF16_TOL
        outs.append(y)
    assert torch.equal(outs[0], outs[1])
