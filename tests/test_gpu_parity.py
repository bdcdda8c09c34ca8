"""GPU parity tests: libqmoe_b200 (through the drop-in qmoe_ns / dense_q modules and the C ABI) against
the CPU oracle (oracle/) and the reference's golden vectors (tests/golden/).

Bars: bit-exact for decode tables, dequantization, layouts, live-neuron sets,
live-group lists and top-k ids; expert and layer outputs within rel-L2 1e-2 of the fp64 oracle (the
fp32-dequantized CPU path). The decode and GEMV kernels accumulate in fp32 as the reference's Triton kernels do
(qmoe_ns.py:4, dense_q.py:8), so they are held to FP32_TOL = 1e-5 of the fp64 oracle, far inside bf16's unit
roundoff (2^-8) that bounds the reference's kernels against each other.
"""
import hashlib

import numpy as np
import pytest
import torch

import vectors as V
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2
BF16_TOL = 2.0 ** -8
FP32_TOL = 1e-5
DEV = "cuda"


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def Q():
    import qmoe_ns
    return qmoe_ns


@pytest.fixture(scope="module")
def D():
    import dense_q
    return dense_q


@pytest.fixture(scope="module")
def synth():
    import qmoe_synth
    return qmoe_synth


@pytest.fixture(scope="module")
def experts(synth):
    """22 synthetic experts (config 0 recipe, p = 7.5%), a token and routing-style coefficients."""
    g = synth.seeded(7, DEV)
    m_hat = synth.unit_dir(g, DEV)
    blk, s2, live = synth.expert_blocks(22, 0.075, m_hat, g, DEV)
    x = synth.tokens(1, m_hat, g, DEV)[0]
    coef = (torch.rand(22, generator=g, device=DEV) * 0.9 + 0.1).float()
    torch.cuda.synchronize()
    return dict(blk=blk, s2=s2.float().contiguous(), live=live, x=x, coef=coef, m_hat=m_hat,
                blk_np=blk.cpu().numpy(), s2_np=s2.cpu().numpy(), x_np=x.float().cpu().numpy(),
                coef_np=coef.cpu().numpy())


@pytest.fixture(scope="module")
def oracle_decode(experts):
    e = experts
    return O.moe_decode(list(e["blk_np"]), e["s2_np"], e["coef_np"], e["x_np"])


# ---------------------------------------------------------------- a1, a11: decode tables, deq
def test_e2m1_table_bit_exact(Q, golden):
    w = torch.arange(256, dtype=torch.uint8, device=DEV).repeat(2).view(1, 512)   # all byte values
    s = torch.full((1, 64), 0x38, dtype=torch.uint8, device=DEV)                   # e4m3 1.0
    out = Q.deq(w, s, 1.0).cpu().numpy()[0]
    e2 = golden["e2m1"]
    ref = np.stack([e2[np.arange(256) & 15], e2[np.arange(256) >> 4]], -1).reshape(-1)
    assert np.array_equal(out[:512].view(np.uint32), ref.view(np.uint32))


def test_e4m3_table_bit_exact(Q, golden):
    w = torch.full((16, 512), 0x22, dtype=torch.uint8, device=DEV)                 # codes 1.0, 1.0
    s = torch.arange(1024, device=DEV).remainder(256).to(torch.uint8).view(16, 64)
    out = Q.deq(w, s, 1.0).cpu().numpy()
    got = out.reshape(16, 64, 16)[:, :, 0].reshape(-1)[:256]
    ref = golden["e4m3"]
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_deq_golden_and_swap(Q, golden):
    b = V.rand_block(1)
    w = torch.from_numpy(b[V.O_UW:V.O_UW + 16 * 512].reshape(16, 512).copy()).to(DEV)
    s = torch.from_numpy(b[V.O_US:V.O_US + 16 * 64].reshape(16, 64).copy()).to(DEV)
    assert np.array_equal(Q.deq(w, s, 0.0123).cpu().numpy().view(np.uint32), golden["deq"].view(np.uint32))
    Q.SWAP = True
    try:
        assert np.array_equal(Q.deq(w, s, 0.0123).cpu().numpy().view(np.uint32), golden["deq_swap"].view(np.uint32))
    finally:
        Q.SWAP = False


def test_block_deq_bit_exact(Q, experts):
    e = experts
    u, d = Q.block_deq(e["blk"][3], e["s2_np"][3])
    ou, od = O.block_deq(e["blk_np"][3], e["s2_np"][3])
    assert np.array_equal(u.cpu().numpy().view(np.uint32), ou.view(np.uint32))
    assert np.array_equal(d.cpu().numpy().view(np.uint32), od.view(np.uint32))


# ---------------------------------------------------------------- a9, a10: layouts
@pytest.mark.parametrize("seed", [2, 3])
def test_layouts_golden(Q, golden, seed):
    m = golden["meta"]
    blk = torch.from_numpy(V.rand_bytes_block(seed)).to(DEV)
    t = Q.to_T(blk)
    assert sha(t.cpu().numpy()) == m[f"to_T_{seed}"]
    assert sha(Q.from_T(blk).cpu().numpy()) == m[f"from_T_{seed}"]
    assert torch.equal(Q.from_T(t), blk)
    g = t.clone().view(1, -1)
    Q.from_T_batch(g)
    assert sha(g.cpu().numpy()) == m[f"from_T_batch_{seed}"]


def test_from_T_fast_batch(Q, experts):
    blk = experts["blk"][:5].contiguous()
    T = blk.clone()
    Q.to_T_batch(T)
    for j in range(5):  # against the oracle's byte permutation
        assert np.array_equal(T[j].cpu().numpy(), O.to_T(experts["blk_np"][j]))
    scratch = torch.empty(5 * 1376256, dtype=torch.uint8, device=DEV)
    back = T.clone()
    Q.from_T_fast(back, scratch)
    assert torch.equal(back, blk)
    assert torch.equal(T[:, :Q.UPB], blk[:, :Q.UPB])


# ---------------------------------------------------------------- a2..a5: decode step
def test_decode_up_and_live_set(Q, experts, oracle_decode):
    e = experts
    K = 22
    sidx = torch.arange(K, dtype=torch.int32, device=DEV)
    h = torch.empty(K, Q.INTER, device=DEV)
    import _qmoe_lib as C
    C.call("qmoe_decode_up", C.ptr(e["blk"]), Q.BLOCK, K, C.ptr(sidx), K, C.ptr(e["s2"]), C.ptr(e["x"]),
           C.dtype_code(e["x"]), C.ptr(h), C.stream_of(h))
    y64, h64, _ = oracle_decode
    hg = h.cpu().numpy()
    assert rel_l2(hg, h64) < FP32_TOL
    # live sets: bit-exact (the synthetic margins are wide), and they match the drawn masks
    assert np.array_equal(hg > 0, h64 > 0)
    # the realized live set is the drawn Bernoulli mask up to the rare live row that comes out negative
    assert int(((hg > 0) != e["live"].cpu().numpy()).sum()) <= 2


def test_live_groups_bit_exact(Q, experts, oracle_decode):
    _, h64, _ = oracle_decode
    h = torch.from_numpy(h64.astype(np.float32)).to(DEV)
    gidx = torch.empty(22, 168, dtype=torch.int32, device=DEV)
    gcnt = torch.empty(22, dtype=torch.int32, device=DEV)
    import _qmoe_lib as C
    C.call("qmoe_live_groups", C.ptr(h), 22, C.ptr(gidx), C.ptr(gcnt), C.stream_of(h))
    og, oc = O.live_groups(h64.astype(np.float32))
    assert np.array_equal(gidx.cpu().numpy(), og)
    assert np.array_equal(gcnt.cpu().numpy(), oc)


def _T_setup(Q, e):
    K = 22
    T = e["blk"].clone()
    Q.to_T_batch(T)
    tab = torch.tensor([T[j].data_ptr() for j in range(K)], dtype=torch.int64, device=DEV)
    bufs = dict(h=torch.empty(K, Q.INTER, device=DEV), part=torch.empty(2, K, Q.LAT, device=DEV),
                gidx=torch.empty(K, 168, dtype=torch.int32, device=DEV), gcnt=torch.empty(K, dtype=torch.int32, device=DEV))
    return T, tab, bufs


def test_moe_decode_groups_parity(Q, experts, oracle_decode):
    e = experts
    K = 22
    T, tab, b = _T_setup(Q, e)
    sidx = torch.arange(K, dtype=torch.int32, device=DEV)
    y = Q.moe_decode_groups(T, sidx, tab, e["s2"], e["coef"], e["x"], b["h"], b["part"], b["gidx"], b["gcnt"])
    torch.cuda.synchronize()
    assert Q.decode_groups_status() == 0
    y64, h64, yj64 = oracle_decode
    yg = y.cpu().numpy()
    err = rel_l2(yg, y64)
    assert err < REL_L2 and err < FP32_TOL, err
    og, oc = O.live_groups(h64.astype(np.float32))
    assert np.array_equal(b["gcnt"].cpu().numpy(), oc)
    assert np.array_equal(b["gidx"].cpu().numpy(), og)
    # determinism: a second call is bit-identical
    y2 = Q.moe_decode_groups(T, sidx, tab, e["s2"], e["coef"], e["x"], b["h"], b["part"], b["gidx"], b["gcnt"])
    assert torch.equal(y, y2)
    # up slots with the UPB stride (the reference's VRAM slots hold only the up half)
    slots_up = T[:, :Q.UPB].contiguous()
    y3 = Q.moe_decode_groups(slots_up, sidx, tab, e["s2"], e["coef"], e["x"], b["h"], b["part"], b["gidx"], b["gcnt"])
    assert torch.equal(y, y3)


def test_down_groups_reference_form(Q, experts, oracle_decode):
    """qmoe_live_groups + qmoe_decode_down_groups with KS = 2 (GROUP_CFG) sum to the fused result."""
    import _qmoe_lib as C
    e = experts
    K = 22
    T, tab, b = _T_setup(Q, e)
    y64, h64, _ = oracle_decode
    h = torch.from_numpy(h64.astype(np.float32)).to(DEV)
    C.call("qmoe_live_groups", C.ptr(h), K, C.ptr(b["gidx"]), C.ptr(b["gcnt"]), C.stream_of(h))
    part = torch.empty(2, K, Q.LAT, device=DEV)
    C.call("qmoe_decode_down_groups", C.ptr(tab), C.ptr(h), C.ptr(b["gidx"]), C.ptr(b["gcnt"]), C.ptr(e["s2"]),
           C.ptr(e["coef"]), K, 2, C.ptr(part), C.stream_of(h))
    y = part.sum((0, 1)).cpu().numpy()
    assert rel_l2(y, y64) < FP32_TOL


def test_zero_skip_vs_full_and_controls(Q, experts, oracle_decode):
    """tests/live_test.py:42-53 and tests/kern_test.py:42-51 patterns: the live-group path equals the
    full orig-layout path; a tab pointing at other experts diverges; slot permutation is invariant."""
    e = experts
    K = 22
    T, tab, b = _T_setup(Q, e)
    sidx = torch.arange(K, dtype=torch.int32, device=DEV)
    h = torch.empty(K, Q.INTER, device=DEV)
    out = torch.empty(K, Q.LAT, device=DEV)
    y_full = Q.moe_decode(e["blk"], sidx, e["s2"], e["coef"], e["x"], h, out)
    y_skip = Q.moe_decode_groups(T, sidx, tab, e["s2"], e["coef"], e["x"], b["h"], b["part"], b["gidx"], b["gcnt"])
    y64 = oracle_decode[0]
    assert rel_l2(y_full.cpu().numpy(), y64) < FP32_TOL
    assert rel_l2(y_skip.cpu().numpy(), y_full.cpu().numpy()) < FP32_TOL
    y_bad = Q.moe_decode_groups(T, sidx, torch.roll(tab, 1), e["s2"], e["coef"], e["x"], b["h"], b["part"],
                                b["gidx"], b["gcnt"])
    assert rel_l2(y_bad.cpu().numpy(), y64) > 0.1
    perm = torch.randperm(K, generator=torch.Generator().manual_seed(3)).to(DEV)
    y_perm = Q.moe_decode_groups(T, sidx[perm].contiguous(), tab[perm].contiguous(), e["s2"][perm].contiguous(),
                                 e["coef"][perm].contiguous(), e["x"], b["h"], b["part"], b["gidx"], b["gcnt"])
    assert rel_l2(y_perm.cpu().numpy(), y_skip.cpu().numpy()) < 1e-5


def test_decode_golden_random_blocks(Q, golden):
    """The golden moe_decode case (random codes, reference block_deq + fp64): both layouts."""
    blocks, s2, coef, x = V.decode_case()
    K = len(blocks)
    blk = torch.from_numpy(np.stack(blocks)).to(DEV)
    s2t = torch.from_numpy(s2).to(DEV)
    ct = torch.from_numpy(coef).to(DEV)
    xt = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    sidx = torch.arange(K, dtype=torch.int32, device=DEV)
    h = torch.empty(K, 2688, device=DEV)
    out = torch.empty(K, 1024, device=DEV)
    y = Q.moe_decode(blk, sidx, s2t, ct, xt, h, out).cpu().numpy()
    gy, gh = golden["decode_y"], golden["decode_h"]
    assert rel_l2(y, gy) < FP32_TOL
    assert rel_l2(h.cpu().numpy(), gh) < FP32_TOL
    # live sets: the kernel's h > 0 equals the fp64 pre-activation's sign on every neuron. The bar excludes only
    # pre-activations within 1e-6 of max|u| of zero (none in this case: the smallest is reported on failure),
    # where fp32 summation order alone could decide the sign.
    hh = h.cpu().numpy()
    u = np.stack([O.deq(b[:V.O_US].reshape(2688, 512), b[V.O_US:V.O_DW].reshape(2688, 64), s2[j, 0]).astype(np.float64)
                  @ x.astype(np.float64) for j, b in enumerate(blocks)])
    flips = int(((hh > 0) != (u > 0)).sum())
    margin = np.abs(u) > 1e-6 * np.abs(u).max()
    assert np.array_equal((hh > 0)[margin], (u > 0)[margin]), f"{flips} live-set flips"
    assert flips == 0, f"{flips} live-set flips; smallest |u|/max|u| = {np.abs(u).min() / np.abs(u).max():.2e}"
    T = blk.clone()
    Q.to_T_batch(T)
    tab = torch.tensor([T[j].data_ptr() for j in range(K)], dtype=torch.int64, device=DEV)
    gidx = torch.empty(K, 168, dtype=torch.int32, device=DEV)
    gcnt = torch.empty(K, dtype=torch.int32, device=DEV)
    part = torch.empty(2, K, 1024, device=DEV)
    y2 = Q.moe_decode_groups(T, sidx, tab, s2t, ct, xt, h, part, gidx, gcnt).cpu().numpy()
    assert rel_l2(y2, gy) < FP32_TOL
    # the fused kernels' live-group lists equal the reference's own glue on the fp64 h (qmoe_ns.py:249-251)
    assert np.array_equal(gidx.cpu().numpy(), golden["decode_gidx"])
    assert np.array_equal(gcnt.cpu().numpy(), golden["decode_gcnt"])


def test_bad_slot_index_gives_nan(Q, experts):
    e = experts
    sidx = torch.arange(22, dtype=torch.int32, device=DEV)
    sidx[5] = 10**6
    h = torch.empty(22, Q.INTER, device=DEV)
    out = torch.empty(22, Q.LAT, device=DEV)
    y = Q.moe_decode(e["blk"], sidx, e["s2"], e["coef"], e["x"], h, out)
    assert torch.isnan(y).all()
    assert not torch.isnan(h[:5]).any() and torch.isnan(h[5]).all()


# ---------------------------------------------------------------- a7, a8: prompt pairs
def test_pairs_golden(Q, golden):
    blocks, pslot, ptok, s2p, coefp, X = V.pairs_case()
    blk = torch.from_numpy(np.stack(blocks)).to(DEV)
    P = len(pslot)
    h = torch.empty(P, 2688, device=DEV)
    out = torch.empty(P, 1024, device=DEV)
    y = Q.moe_pairs(blk, torch.from_numpy(pslot).to(DEV), torch.from_numpy(ptok).to(DEV),
                    torch.from_numpy(s2p).to(DEV), torch.from_numpy(coefp).to(DEV),
                    torch.from_numpy(X).to(DEV).to(torch.bfloat16), h, out)
    assert rel_l2(y.cpu().numpy(), golden["pairs_out"]) < FP32_TOL


def test_pairs_vs_step(Q, experts):
    """tests/pairs_test.py:34-50: pairs + fixed-order combine equal per-token decode."""
    e = experts
    Tn, NB = 7, 22
    g = torch.Generator(device=DEV)
    g.manual_seed(11)
    import qmoe_synth as S
    X = S.tokens(Tn, e["m_hat"], g, DEV)
    sel = torch.stack([torch.randperm(NB, generator=torch.Generator().manual_seed(t))[:8] for t in range(Tn)]).to(DEV)
    w = torch.rand(Tn, 8, generator=g, device=DEV)
    t_i = torch.arange(Tn, device=DEV).repeat_interleave(8)
    k_i = torch.arange(8, device=DEV).repeat(Tn)
    b_i = sel[t_i, k_i]
    h = torch.empty(Tn * 8, 2688, device=DEV)
    out = torch.empty(Tn * 8, 1024, device=DEV)
    y = Q.moe_pairs(e["blk"], b_i.int().contiguous(), t_i.int().contiguous(), e["s2"][b_i].contiguous(),
                    w[t_i, k_i].float().contiguous(), X, h, out)
    Yd = torch.zeros(Tn, 8, 1024, device=DEV)
    Yd[t_i, k_i] = y
    comb = Yd.sum(1)
    for t in range(Tn):
        ref = Q.moe_decode(e["blk"], sel[t].int().contiguous(), e["s2"][sel[t]].contiguous(), w[t].contiguous(), X[t],
                           torch.empty(8, 2688, device=DEV), torch.empty(8, 1024, device=DEV))
        # two kernel paths (pairs GEMV vs decode up/down), both fp32: they differ only in summation order
        assert rel_l2(comb[t].cpu().numpy(), ref.cpu().numpy()) < FP32_TOL
    # T-layout slots (qmoe_ns.moe_pairs_T) give the same pairs
    T = e["blk"].clone()
    Q.to_T_batch(T)
    y2 = Q.moe_pairs_T(T, b_i.int().contiguous(), t_i.int().contiguous(), e["s2"][b_i].contiguous(),
                       w[t_i, k_i].float().contiguous(), X, torch.empty_like(h), torch.empty_like(out))
    assert torch.equal(y2, y)


# ---------------------------------------------------------------- a12..a15: dense
@pytest.mark.parametrize("fmt,seed", [("fp8", 400), ("nvfp4", 401)])
def test_dense_golden(D, golden, fmt, seed):
    w, sc, s, x = V.dense_case(fmt, seed)
    N = w.shape[0]
    K = w.shape[1] * (2 if fmt == "nvfp4" else 1)
    q = {"fmt": fmt, "w": torch.from_numpy(w).to(DEV), "s": torch.tensor([s], device=DEV), "N": N, "K": K}
    if sc is not None:
        q["sc"] = torch.from_numpy(sc).to(DEV)
    o16 = torch.empty(N, K, dtype=torch.bfloat16, device=DEV)
    D.dequant_rows(q, 0, N, o16)
    assert np.array_equal(o16.view(torch.int16).cpu().numpy().view(np.uint16), golden[f"dense_{fmt}_bf16"])
    o32 = torch.empty(N, K, dtype=torch.float32, device=DEV)
    D.dequant_rows(q, 0, N, o32)
    assert np.array_equal(o32.cpu().numpy().view(np.uint32), golden[f"dense_{fmt}_w32"].view(np.uint32))
    xt = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    y = D.gemv_mb(q, xt).cpu().numpy()
    assert rel_l2(y, golden[f"dense_{fmt}_y"]) < FP32_TOL
    y1 = D.gemv(q, xt[0]).cpu().numpy()
    assert rel_l2(y1, golden[f"dense_{fmt}_y"][0]) < FP32_TOL


DENSE_SHAPES = [("fp8", 4096, 4096), ("fp8", 12288, 4096), ("fp8", 4096, 8192), ("fp8", 10304, 2688),
                ("fp8", 2688, 4096), ("nvfp4", 2688, 4096), ("nvfp4", 4096, 2688), ("nvfp4", 3712, 2688),
                ("nvfp4", 2688, 3712)]


@pytest.mark.parametrize("fmt,N,K", DENSE_SHAPES)
def test_dense_gemv_shapes(D, synth, fmt, N, K):
    g = synth.seeded(N + K, DEV)
    wf = torch.randn(N, K, generator=g, device=DEV) * 0.02
    if fmt == "fp8":
        codes, s = synth.quantize_fp8(wf)
        q = {"fmt": "fp8", "w": codes, "s": s.to(DEV), "N": N, "K": K}
        sc_np = None
    else:
        codes, sc, s2 = synth.quantize_nvfp4(wf)
        q = {"fmt": "nvfp4", "w": codes, "sc": sc, "s": s2.reshape(1), "N": N, "K": K}
        sc_np = sc.cpu().numpy()
    x = torch.randn(4, K, generator=g, device=DEV).to(torch.bfloat16)
    ref = O.dense(fmt, q["w"].cpu().numpy(), sc_np, float(q["s"]), N, K, x.float().cpu().numpy())
    for M in (1, 2, 3, 4):
        y = D.qlinear(q, x[:M].float()).float().cpu().numpy() if M > 1 else D.gemv(q, x[0]).cpu().numpy()[None]
        assert rel_l2(y, ref[:M]) < FP32_TOL, (M, rel_l2(y, ref[:M]))
    # M > MB_MAX: exact dequantization + cuBLAS (bf16 operands, as the reference's dequant + F.linear)
    y5 = D.qlinear(q, torch.cat([x, x[:1]]).to(torch.bfloat16)).float().cpu().numpy()
    assert rel_l2(y5[:4], ref) < 2e-2


def test_dense_lm_head_parity_sampled(D, synth):
    """131072 x 4096 FP8 (the lm_head of config 2): rows checked against the oracle on a sample."""
    N, K = 131072, 4096
    g = synth.seeded(5, DEV)
    codes = torch.randint(0, 0x7E, (N, K), generator=g, device=DEV, dtype=torch.int32).to(torch.uint8)
    codes |= (torch.randint(0, 2, (N, K), generator=g, device=DEV, dtype=torch.int32) << 7).to(torch.uint8)
    q = {"fmt": "fp8", "w": codes, "s": torch.tensor([0.00123], device=DEV), "N": N, "K": K}
    x = torch.randn(K, generator=g, device=DEV).to(torch.bfloat16)
    y = D.gemv(q, x)
    rows = torch.arange(0, N, 977, device=DEV)
    ref = O.dense("fp8", codes[rows].cpu().numpy(), None, 0.00123, len(rows), K, x.float().cpu().numpy()[None])[0]
    assert rel_l2(y[rows].cpu().numpy(), ref) < FP32_TOL


def test_decode_groups_large_K_two_kernel_path(Q, experts, oracle_decode):
    """K > 64 takes the up / down_groups kernel pair; 3 copies of the 22 experts (K = 66) with a third
    of the coefficients each must give the K = 22 result."""
    e = experts
    T, tab, _ = _T_setup(Q, e)
    K = 66
    sidx = torch.arange(22, dtype=torch.int32, device=DEV).repeat(3)
    tab3 = tab.repeat(3)
    s2 = e["s2"].repeat(3, 1).contiguous()
    coef = (e["coef"] / 3).repeat(3).contiguous()
    h = torch.empty(K, Q.INTER, device=DEV)
    part = torch.empty(2, K, Q.LAT, device=DEV)
    gidx = torch.empty(K, 168, dtype=torch.int32, device=DEV)
    gcnt = torch.empty(K, dtype=torch.int32, device=DEV)
    y = Q.moe_decode_groups(T, sidx, tab3, s2, coef, e["x"], h, part, gidx, gcnt)
    assert rel_l2(y.cpu().numpy(), oracle_decode[0]) < FP32_TOL
    og, oc = O.live_groups(h.cpu().numpy())
    assert np.array_equal(gidx.cpu().numpy(), og) and np.array_equal(gcnt.cpu().numpy(), oc)


@pytest.mark.parametrize("K", [1, 4, 8, 9, 19, 25, 31, 33, 38, 49, 75, 148, 150])
def test_decode_groups_K_range(Q, experts, K):
    """moe_decode_groups for K experts (entry j -> expert j mod 22). Up to the SM count (148) the fused layer kernel
    runs with S = 8, 7, 6, 4, 3, 2 or 1 CTAs per expert (each S is taken by one of these K); K = 150 takes the
    up kernel + arrival-counter down kernel. y and the per-expert outputs within 1e-5 of the fp64 oracle, gidx /
    gcnt the exact compaction of the kernel's h."""
    e = experts
    T, tab, _ = _T_setup(Q, e)
    idx = torch.arange(K, device=DEV) % 22
    coef = (torch.rand(K, generator=torch.Generator(device=DEV).manual_seed(K), device=DEV) + 0.1).contiguous()
    h = torch.empty(K, Q.INTER, device=DEV)
    part = torch.empty(2, K, Q.LAT, device=DEV)
    gidx = torch.empty(K, 168, dtype=torch.int32, device=DEV)
    gcnt = torch.empty(K, dtype=torch.int32, device=DEV)
    y = Q.moe_decode_groups(T, idx.to(torch.int32).contiguous(), tab[idx].contiguous(), e["s2"][idx].contiguous(), coef,
                            e["x"], h, part, gidx, gcnt)
    torch.cuda.synchronize()
    assert Q.decode_groups_status() == 0
    ii = idx.cpu().numpy()
    y64, _, yj64 = O.moe_decode([e["blk_np"][i] for i in ii], e["s2_np"][ii], coef.cpu().numpy(), e["x_np"])
    assert rel_l2(y.cpu().numpy(), y64) < FP32_TOL
    assert rel_l2(part[0].cpu().numpy(), yj64) < FP32_TOL
    og, oc = O.live_groups(h.cpu().numpy())
    assert np.array_equal(gidx.cpu().numpy(), og) and np.array_equal(gcnt.cpu().numpy(), oc)


def test_decode_groups_graph_capture_and_determinism(Q, experts, oracle_decode):
    e = experts
    K = 22
    T, tab, b = _T_setup(Q, e)
    sidx = torch.arange(K, dtype=torch.int32, device=DEV)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        y0 = Q.moe_decode_groups(T, sidx, tab, e["s2"], e["coef"], e["x"], b["h"], b["part"], b["gidx"], b["gcnt"])
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            yg = Q.moe_decode_groups(T, sidx, tab, e["s2"], e["coef"], e["x"], b["h"], b["part"], b["gidx"],
                                     b["gcnt"])
        outs = []
        for _ in range(5):
            g.replay()
            outs.append(yg.clone())
    st.synchronize()
    for o in outs:
        assert torch.equal(o, y0)      # bit-identical replays
    assert rel_l2(y0.cpu().numpy(), oracle_decode[0]) < FP32_TOL


def test_copy_async_and_decode_with_host_y(Q, experts):
    """qmoe_copy_async moves small records between pinned host memory and the device inside the kernel chain
    (16-byte words with odd tails, and bytes when an end is unaligned) and writes nothing outside the range;
    qmoe_decode_groups with y in pinned host memory (the per-layer host round trip of the bench's e2e leg,
    inputs staged by qmoe_copy_async) gives the device-resident result bit for bit."""
    import _qmoe_lib as C
    lib = C.lib()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(5)
    for n, soff, doff in ((1, 0, 0), (15, 0, 0), (2576, 0, 0), (100003, 0, 0), (4099, 3, 1), (64, 16, 5)):
        src = torch.randint(0, 256, (n + soff,), dtype=torch.uint8, generator=g).pin_memory()
        dev = torch.zeros(n + 32, dtype=torch.uint8, device=DEV)
        back = torch.zeros(n, dtype=torch.uint8).pin_memory()
        assert lib.qmoe_copy_async(dev.data_ptr() + doff, src.data_ptr() + soff, n, st) == 0
        assert lib.qmoe_copy_async(back.data_ptr(), dev.data_ptr() + doff, n, st) == 0
        torch.cuda.synchronize()
        assert torch.equal(back, src[soff:])
        assert int(dev[:doff].sum()) == 0 and int(dev[doff + n:].sum()) == 0
    assert lib.qmoe_copy_async(0, 0, 0, st) == 0              # nothing to do
    assert lib.qmoe_copy_async(0, src.data_ptr(), 8, st) == 5  # QMOE_ERR_NULL

    e = experts
    K = 22
    T, tab, b = _T_setup(Q, e)
    sidx = torch.arange(K, dtype=torch.int32, device=DEV)
    y_dev = Q.moe_decode_groups(T, sidx, tab, e["s2"], e["coef"], e["x"], b["h"], b["part"], b["gidx"], b["gcnt"])
    x_host = e["x"].cpu().pin_memory()
    x_dev = torch.empty_like(e["x"])
    y_host = torch.full((Q.LAT,), float("nan")).pin_memory()
    ws = torch.zeros(int(lib.qmoe_decode_groups_workspace_bytes(K)), dtype=torch.uint8, device=DEV)
    assert lib.qmoe_copy_async(x_dev.data_ptr(), x_host.data_ptr(), x_host.numel() * 2, st) == 0
    rc = lib.qmoe_decode_groups(T.data_ptr(), T.stride(0), T.shape[0], sidx.data_ptr(), tab.data_ptr(),
                                e["s2"].data_ptr(), e["coef"].data_ptr(), x_dev.data_ptr(), C.dtype_code(x_dev), K,
                                b["h"].data_ptr(), b["gidx"].data_ptr(), b["gcnt"].data_ptr(), b["part"].data_ptr(),
                                y_host.data_ptr(), ws.data_ptr(), ws.numel(), st)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(y_host, y_dev.cpu())


@pytest.mark.parametrize("xdt", [torch.float16, torch.float32])
def test_activation_dtypes(Q, D, synth, experts, xdt):
    """f16 and fp32 activations (the other two x dtypes of the C ABI) through the decode layer (the fused kernel
    at K = 22 and the two-kernel path at K = 150; fp32 activations run separate kernel instantiations that keep
    x in fp32), the prefill grouped GEMM, and the FP8 / NVFP4 GEMVs, each against the fp64 oracle evaluated on the
    very values passed in."""
    e = experts
    g = synth.seeded(77, DEV)
    x = e["x"].float()
    if xdt == torch.float32:
        x = x + 1e-3 * torch.randn(x.shape, generator=g, device=DEV)   # values bf16 and f16 cannot hold
    x = x.to(xdt)
    x_np = x.float().cpu().numpy()
    T, tab, _ = _T_setup(Q, e)
    for K in (22, 150):
        idx = torch.arange(K, device=DEV) % 22
        coef = (torch.rand(K, generator=g, device=DEV) + 0.1).contiguous()
        h = torch.empty(K, Q.INTER, device=DEV)
        part = torch.empty(2, K, Q.LAT, device=DEV)
        gidx = torch.empty(K, 168, dtype=torch.int32, device=DEV)
        gcnt = torch.empty(K, dtype=torch.int32, device=DEV)
        y = Q.moe_decode_groups(T, idx.to(torch.int32).contiguous(), tab[idx].contiguous(), e["s2"][idx].contiguous(),
                                coef, x, h, part, gidx, gcnt)
        ii = idx.cpu().numpy()
        y64, _, _ = O.moe_decode([e["blk_np"][i] for i in ii], e["s2_np"][ii], coef.cpu().numpy(), x_np)
        assert rel_l2(y.cpu().numpy(), y64) < FP32_TOL, (K, rel_l2(y.cpu().numpy(), y64))

    # prefill: 8 tokens (scaled copies of x) routed to 6 of the 22 orig-layout experts each
    Tt, k = 8, 6
    rng = np.random.default_rng(3)
    ids = np.stack([rng.permutation(22)[:k] for _ in range(Tt)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, (Tt, k)).astype(np.float32)
    X = torch.stack([x.float() * (0.5 + 0.15 * i) for i in range(Tt)]).to(xdt)
    yp = Q.moe_prefill(e["blk"], torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV), e["s2"], X,
                       layout_T=False)
    pslot = ids.reshape(-1)
    ptok = np.repeat(np.arange(Tt, dtype=np.int32), k)
    ref = O.pairs(list(e["blk_np"]), pslot, ptok, e["s2_np"][pslot], w.reshape(-1), X.float().cpu().numpy())
    assert rel_l2(yp.cpu().numpy(), ref.reshape(Tt, k, -1).sum(1)) < 2.0 ** -8
    assert Q.prefill_status() == 0

    # dense GEMVs at M = 1
    for fmt, N, Kd in (("fp8", 4096, 4096), ("nvfp4", 2688, 4096)):
        wf = torch.randn(N, Kd, generator=g, device=DEV) * 0.02
        if fmt == "fp8":
            codes, s = synth.quantize_fp8(wf)
            q = {"fmt": "fp8", "w": codes, "s": s.to(DEV), "N": N, "K": Kd}
            sc_np = None
        else:
            codes, sc, s2 = synth.quantize_nvfp4(wf)
            q = {"fmt": "nvfp4", "w": codes, "sc": sc, "s": s2.reshape(1), "N": N, "K": Kd}
            sc_np = sc.cpu().numpy()
        xv = torch.randn(Kd, generator=g, device=DEV).to(xdt)
        ref = O.dense(fmt, q["w"].cpu().numpy(), sc_np, float(q["s"]), N, Kd, xv.float().cpu().numpy()[None])[0]
        assert rel_l2(D.gemv(q, xv).cpu().numpy(), ref) < FP32_TOL, fmt


def test_nvfp4_gemv_bf16_epilogues(D, synth):
    """dq_gemv_nvfp4_bf16: the bf16 cast, bf16(relu(bf16(v))^2) and bf16(bf16(v) + residual) equal torch's bf16
    operators applied to dq_gemv_nvfp4's fp32 result, bit for bit (M = 1 and 2)."""
    import _qmoe_lib as C
    g = synth.seeded(808, DEV)
    N, K = 2688, 4096
    codes, sc, s2 = synth.quantize_nvfp4(torch.randn(N, K, generator=g, device=DEV) * 0.02)
    q = {"fmt": "nvfp4", "w": codes, "sc": sc, "s": s2.reshape(1), "N": N, "K": K}
    for M in (1, 2):
        x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
        v = D.gemv_mb(q, x) if M > 1 else D.gemv(q, x[0]).view(1, N)
        res = torch.randn(M, N, generator=g, device=DEV).to(torch.bfloat16)
        u = torch.relu(v.to(torch.bfloat16))
        expect = {0: v.to(torch.bfloat16), 1: u * u, 2: v.to(torch.bfloat16) + res}
        for ep in (0, 1, 2):
            y = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
            C.call("dq_gemv_nvfp4_bf16", C.ptr(codes), C.ptr(sc), C.ptr(q["s"]), C.ptr(x), C.dtype_code(x), M, N, K,
                   ep, C.ptr(res) if ep == 2 else None, C.ptr(y), C.stream_of(x))
            assert torch.equal(y, expect[ep]), (M, ep)


@pytest.mark.parametrize("ne,k", [(37, 5), (512, 1), (512, 22), (512, 32), (1024, 22)])
def test_route_decode_shapes_and_ties(ne, k):
    """qmoe_route_decode on random fp32 logits for expert counts that are not multiples of 32 and the limits
    (1024 experts, top-32): the chosen set and its weights are those of torch (sigmoid, + bias, top-k, x scaling),
    the order is by decreasing choice, and the store rows, block addresses and s2 rows follow the slot base.
    Equal choices go to the lower expert id."""
    import _qmoe_lib as C
    g = torch.Generator(device=DEV).manual_seed(ne * 100 + k)
    logits = torch.randn(ne, generator=g, device=DEV) * 3
    bias = torch.randn(ne, generator=g, device=DEV) * 0.01
    s2 = torch.rand(ne, 2, generator=g, device=DEV)
    blocks = torch.empty(4, 64, dtype=torch.uint8, device=DEV)      # only addresses are formed from it
    outs = dict(ids=torch.empty(k, dtype=torch.int64, device=DEV), sidx=torch.empty(k, dtype=torch.int32, device=DEV),
                tab=torch.empty(k, dtype=torch.int64, device=DEV), s2=torch.empty(k, 2, device=DEV),
                coef=torch.empty(k, device=DEV))

    def run(lg):
        C.call("qmoe_route_decode", C.ptr(lg), C.ptr(bias), ne, k, 2.5, 7, C.ptr(blocks), 1000, C.ptr(s2),
               C.ptr(outs["ids"]), C.ptr(outs["sidx"]), C.ptr(outs["tab"]), C.ptr(outs["s2"]), C.ptr(outs["coef"]),
               C.stream_of(lg))
        torch.cuda.synchronize()
        return {n: t.clone() for n, t in outs.items()}

    o = run(logits)
    score = logits.sigmoid()
    choice = score + bias
    ref = torch.topk(choice, k, sorted=False)[1]
    assert set(o["ids"].tolist()) == set(ref.tolist())
    assert torch.equal(o["coef"], score[o["ids"]] * 2.5)
    assert torch.all(choice[o["ids"]][:-1] >= choice[o["ids"]][1:])
    assert torch.equal(o["sidx"], (o["ids"] + 7).to(torch.int32))
    assert torch.equal(o["tab"], blocks.data_ptr() + (o["ids"] + 7) * 1000)
    assert torch.equal(o["s2"], s2[o["ids"]])
    # ties: every logit equal and no bias -> the k lowest ids, in order
    flat = torch.zeros(ne, device=DEV)
    bias.zero_()
    o = run(flat)
    assert o["ids"].tolist() == list(range(k))


@pytest.mark.parametrize("N,K,M", [(4096, 1024, 1), (1024, 4096, 1), (1000, 4104, 3)])
def test_bf16_gemv(N, K, M):
    """dq_gemv_bf16 (bf16 weights widened exactly, fp32 accumulation, bf16 result) against the fp64 product rounded
    to bf16: within one bf16 rounding (rel-L2 <= 2^-8, nearly every element equal); its relu^2 and residual
    epilogues equal torch's bf16 operators applied to its plain result, bit for bit."""
    import _qmoe_lib as C
    g = torch.Generator(device=DEV).manual_seed(N + K + M)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    res = torch.randn(M, N, generator=g, device=DEV).to(torch.bfloat16)
    outs = {}
    for ep in (0, 1, 2):
        y = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        C.call("dq_gemv_bf16", C.ptr(w), C.ptr(x), C.dtype_code(x), M, N, K, ep, C.ptr(res) if ep == 2 else None,
               C.ptr(y), C.stream_of(x))
        outs[ep] = y
    ref = (x.double() @ w.double().t())
    y0 = outs[0]
    assert rel_l2(y0.float().cpu().numpy(), ref.cpu().numpy()) < 2.0 ** -8
    assert (y0 == ref.to(torch.bfloat16)).float().mean().item() > 0.99
    u = torch.relu(y0)
    assert torch.equal(outs[1], u * u)
    assert torch.equal(outs[2], y0 + res)
    # fp32 x rounded to bf16 as it is read (x_dtype 3) = the bf16 cast of x before the call
    xf = x.float() + 1e-3 * torch.randn(M, K, generator=g, device=DEV)
    y3 = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    yc = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    xc = xf.to(torch.bfloat16)
    C.call("dq_gemv_bf16", C.ptr(w), C.ptr(xf), 3, M, N, K, 0, None, C.ptr(y3), C.stream_of(x))
    C.call("dq_gemv_bf16", C.ptr(w), C.ptr(xc), C.dtype_code(xc), M, N, K, 0, None, C.ptr(yc), C.stream_of(x))
    assert torch.equal(y3, yc)


def test_new_entry_points_at_their_edges(D, synth):
    """The bf16-result GEMVs at M = 3 and 4 and with f16 / fp32 vectors, and the routing kernel with one expert and
    top-1: each against the same computation by torch on the same values."""
    import _qmoe_lib as C
    g = synth.seeded(909, DEV)
    N, K = 512, 1024
    codes, sc, s2 = synth.quantize_nvfp4(torch.randn(N, K, generator=g, device=DEV) * 0.02)
    q = {"fmt": "nvfp4", "w": codes, "sc": sc, "s": s2.reshape(1), "N": N, "K": K}
    for M in (3, 4):
        x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
        v = D.gemv_mb(q, x)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        C.call("dq_gemv_nvfp4_bf16", C.ptr(codes), C.ptr(sc), C.ptr(q["s"]), C.ptr(x), C.dtype_code(x), M, N, K, 1,
               None, C.ptr(y), C.stream_of(x))
        u = torch.relu(v.to(torch.bfloat16))
        assert torch.equal(y, u * u), M
    wb = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    for xdt in (torch.float16, torch.float32):
        x = torch.randn(2, K, generator=g, device=DEV).to(xdt)
        y = torch.empty(2, N, dtype=torch.bfloat16, device=DEV)
        C.call("dq_gemv_bf16", C.ptr(wb), C.ptr(x), C.dtype_code(x), 2, N, K, 0, None, C.ptr(y), C.stream_of(x))
        ref = (x.double() @ wb.double().t())
        assert rel_l2(y.float().cpu().numpy(), ref.cpu().numpy()) < 2.0 ** -8, xdt
    logits = torch.randn(1, device=DEV)
    bias = torch.zeros(1, device=DEV)
    s2r = torch.rand(1, 2, device=DEV)
    blocks = torch.empty(1, 16, dtype=torch.uint8, device=DEV)
    o = dict(ids=torch.empty(1, dtype=torch.int64, device=DEV), sidx=torch.empty(1, dtype=torch.int32, device=DEV),
             tab=torch.empty(1, dtype=torch.int64, device=DEV), s2=torch.empty(1, 2, device=DEV),
             coef=torch.empty(1, device=DEV))
    C.call("qmoe_route_decode", C.ptr(logits), C.ptr(bias), 1, 1, 1.0, 0, C.ptr(blocks), 16, C.ptr(s2r),
           C.ptr(o["ids"]), C.ptr(o["sidx"]), C.ptr(o["tab"]), C.ptr(o["s2"]), C.ptr(o["coef"]), C.stream_of(logits))
    torch.cuda.synchronize()
    assert int(o["ids"]) == 0 and int(o["sidx"]) == 0 and int(o["tab"]) == blocks.data_ptr()
    assert torch.equal(o["coef"], logits.sigmoid()) and torch.equal(o["s2"], s2r)
