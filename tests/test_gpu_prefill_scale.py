"""Prefill parity at BASELINE config 3 scale: one 512-expert layer (config 0 recipe), tokens drawn as in config 0
and routed top-22 of 512 by the synthetic router, T = 64, 2048 and 8192 - the calls bench.py times - through the
drop-in qmoe_ns.moe_prefill (qmoe_prefill_grouped: routing sort, NVFP4 planes, block-scaled tcgen05 up/down GEMMs,
k-order combine), replacing the prompt path of nem_super.py:335-348 (moe_pairs arithmetic, qmoe_ns.py:79-133).

Checked per token against the fp64 oracle (pairs + k-order combine) at rel-L2 <= 2^-8 on a sample: every token of
one expert with at least one full 128-pair tile (its first tile full, the rest in further tiles) plus tokens
spread over the prompt (all tokens at T = 64). The orig and T layouts must give bit-identical outputs (the T
layout's down halves are converted inside the call), and the device status word must stay clear.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 2.0 ** -8
DEV = "cuda"
NE, K = 512, 22


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def layer512():
    import qmoe_ns as Q
    import qmoe_synth as S
    g = S.seeded(77, DEV)
    m_hat = S.unit_dir(g, DEV)
    router = S.router(g, DEV)
    store = torch.empty(NE, S.BLOCK, dtype=torch.uint8, device=DEV)
    s2 = torch.empty(NE, 2, dtype=torch.float32, device=DEV)
    for e0 in range(0, NE, 32):
        blk, s2b, _ = S.expert_blocks(32, 0.0875, m_hat, g, DEV)
        store[e0:e0 + 32].copy_(blk)
        s2[e0:e0 + 32] = s2b
        del blk
    storeT = store.clone()
    Q.to_T_batch(storeT)
    torch.cuda.synchronize()
    return dict(store=store, storeT=storeT, s2=s2, m_hat=m_hat, router=router, blocks=list(store.cpu().numpy()),
                s2_np=s2.cpu().numpy())


def _sample(ids, T):
    """Every token of the expert with the fewest pairs among those with >= 128 (one full tile at least), plus
    tokens spread over the prompt; all tokens when T <= 64."""
    if T <= 64:
        return np.arange(T), None
    counts = np.bincount(ids.ravel(), minlength=NE)
    full = np.nonzero(counts >= 128)[0]
    e = int(full[np.argmin(counts[full])]) if len(full) else int(counts.argmax())
    tok = np.nonzero((ids == e).any(1))[0]
    spread = np.linspace(0, T - 1, 64).round().astype(np.int64)
    return np.unique(np.concatenate([tok, spread])), (e, int(counts[e]))


@pytest.mark.parametrize("T", [64, 2048, 8192])
def test_prefill_config3_scale(layer512, T):
    import qmoe_ns as Q
    import qmoe_synth as S
    L = layer512
    X = S.tokens(T, L["m_hat"], S.seeded(1000 + T, DEV), DEV)
    ids, w = S.route(X, *L["router"])
    ids = ids.to(torch.int32).contiguous()
    w = w.float().contiguous()
    y = Q.moe_prefill(L["store"], ids, w, L["s2"], X, layout_T=False)
    yT = Q.moe_prefill(L["storeT"], ids, w, L["s2"], X, layout_T=True)
    torch.cuda.synchronize()
    assert Q.prefill_status() == 0
    assert torch.equal(y, yT)
    ids_np = ids.cpu().numpy()
    sample, tiled = _sample(ids_np, T)
    if T >= 2048:
        assert tiled is not None and tiled[1] >= 128, tiled   # a full 128-pair tile is among the tokens checked
    ref = O.prefill(L["blocks"], L["s2_np"], ids_np[sample], w.cpu().numpy()[sample], X.float().cpu().numpy()[sample])
    got = y.cpu().numpy()[sample]
    errs = [rel_l2(got[i], ref[i]) for i in range(len(sample))]
    assert len(sample) >= min(T, 128)
    assert max(errs) < BF16_TOL, (max(errs), int(sample[int(np.argmax(errs))]))
    assert rel_l2(got, ref) < BF16_TOL
