"""qmoe_decode_groups_static — the decode-step layer for callers that cannot allocate device memory (hosts
whose HBM is already committed to their own pool, code inside a CUDA graph capture that refuses
allocation calls, foreign-language hosts that only pass pointers through). It keeps its scratch in a
static device array inside the library instead of a caller workspace.

Checked here through the C ABI against the workspace entry point qmoe_decode_groups on the same inputs. Both
run the same kernels with the same fixed summation order, so every output must be bit-identical:
  - two calls in a row (the second finds the first call's leftovers in the shared array), K = 22 (the fused
    layer kernel, 6 CTAs per expert);
  - K = 80 (one CTA per expert); also within 1e-5 of the fp64 oracle;
  - the workspace entry point at K = 150 (more experts than SMs: the up kernel + arrival-counter down kernel)
    on a workspace whose arrival counters hold garbage: the up kernel must clear them, or the down kernel's
    last-arriving CTA never sums y;
  - a misaligned tab entry: that expert's part row and y are NaN, the static status word reads
    QMOE_ERR_ALIGN through qmoe_decode_groups_static_status and clears, and the next call is clean;
  - K above the static limit is refused before any work.
The file name sorts last so that a run stopping at the first failure has run every other test.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
DEV = "cuda"
ERR_ALIGN = 2


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def layer():
    import qmoe_ns as Q
    import qmoe_synth as S
    g = S.seeded(31, DEV)
    m_hat = S.unit_dir(g, DEV)
    NB = 22
    blk, s2, _ = S.expert_blocks(NB, 0.075, m_hat, g, DEV)
    orig = blk.cpu().numpy()
    Q.to_T_batch(blk)
    xs = S.tokens(2, m_hat, g, DEV)
    coef = (torch.rand(80, generator=g, device=DEV) * 5).float()
    tab = torch.tensor([blk[j].data_ptr() for j in range(NB)], dtype=torch.int64, device=DEV)
    torch.cuda.synchronize()
    return dict(blk=blk, orig=orig, s2=s2.float().contiguous(), xs=xs, coef=coef, tab=tab, NB=NB)


def _case(L, K):
    """K routed entries over the NB experts (entry j -> expert j mod NB)."""
    sidx = (torch.arange(K, device=DEV) % L["NB"]).to(torch.int32)
    return dict(sidx=sidx, tab=L["tab"][sidx.long()].contiguous(), s2=L["s2"][sidx.long()].contiguous(),
                coef=L["coef"][:K].contiguous(), K=K)


def _bufs(K):
    return dict(h=torch.empty(K, 2688, device=DEV), part=torch.empty(K, 1024, device=DEV),
                gidx=torch.empty(K, 168, dtype=torch.int32, device=DEV), gcnt=torch.empty(K, dtype=torch.int32, device=DEV),
                y=torch.empty(1024, device=DEV))


def _call(name, L, c, x, b, extra=()):
    import _qmoe_lib as C
    blk = L["blk"]
    args = [C.ptr(blk), blk.stride(0), blk.shape[0], C.ptr(c["sidx"]), C.ptr(c["tab"]), C.ptr(c["s2"]),
            C.ptr(c["coef"]), C.ptr(x), C.dtype_code(x), c["K"], C.ptr(b["h"]), C.ptr(b["gidx"]), C.ptr(b["gcnt"]),
            C.ptr(b["part"]), C.ptr(b["y"])]
    return getattr(C.lib(), name)(*args, *extra, C.stream_of(x))


def _static_status(clear):
    import _qmoe_lib as C
    return int(C.lib().qmoe_decode_groups_static_status(int(clear), C.stream_of()))


def _workspace(K):
    import _qmoe_lib as C
    return torch.zeros(int(C.lib().qmoe_decode_groups_workspace_bytes(K)), dtype=torch.uint8, device=DEV)


def _same(a, b):
    for k in ("y", "h", "part", "gidx", "gcnt"):
        assert torch.equal(a[k], b[k]), k


@pytest.mark.parametrize("K", [22, 80])
def test_static_entry_point_matches_workspace_entry_point(layer, K):
    import _qmoe_lib as C
    L = layer
    c = _case(L, K)
    ws = _workspace(K)
    assert _static_status(True) in (0, ERR_ALIGN)   # start from a clear status word
    for call in range(2):   # two calls in a row, different tokens
        x = L["xs"][call]
        ref = _bufs(K)
        assert _call("qmoe_decode_groups", L, c, x, ref, (C.ptr(ws), ws.numel())) == 0
        got = _bufs(K)
        assert _call("qmoe_decode_groups_static", L, c, x, got) == 0
        torch.cuda.synchronize()
        _same(got, ref)
        assert torch.isfinite(got["y"]).all()
    assert _static_status(False) == 0
    if K == 80:   # the global-metadata path of the up kernel against the fp64 oracle
        y64, _, _ = O.moe_decode([L["orig"][j % L["NB"]] for j in range(K)], c["s2"].cpu().numpy(),
                                 c["coef"].cpu().numpy(), L["xs"][1].float().cpu().numpy())
        assert rel_l2(got["y"].cpu().numpy(), y64) < FP32_TOL


def test_workspace_counters_left_dirty_are_cleared(layer):
    """K = 150 (more experts than SMs: the up kernel + arrival-counter down kernel, whose counters live in the
    workspace): the counters (bytes 64..95) filled with garbage, the status word zero. The up kernel clears them
    before the down kernel counts, so the result equals that of a clean workspace."""
    import _qmoe_lib as C
    L = layer
    K = 150
    L = dict(layer, coef=(torch.arange(K, device=DEV, dtype=torch.float32) % 7 + 1) / 7)
    c = _case(L, K)
    x = L["xs"][0]
    clean, dirty = _bufs(K), _bufs(K)
    ws = _workspace(K)
    assert _call("qmoe_decode_groups", L, c, x, clean, (C.ptr(ws), ws.numel())) == 0
    ws2 = _workspace(K)
    ws2[64:96] = 0x5A
    assert _call("qmoe_decode_groups", L, c, x, dirty, (C.ptr(ws2), ws2.numel())) == 0
    torch.cuda.synchronize()
    _same(dirty, clean)
    assert int(C.lib().qmoe_workspace_status(C.ptr(ws2), 1, C.stream_of(x))) == 0


def test_static_bad_tab_entry_sets_and_clears_status(layer):
    L = layer
    c = _case(L, 22)
    x = L["xs"][0]
    assert _static_status(True) in (0, ERR_ALIGN)
    bad = dict(c)
    bad["tab"] = c["tab"].clone()
    bad["tab"][3] += 8                       # not 16-byte aligned: the down kernel reads nothing for expert 3
    b = _bufs(22)
    assert _call("qmoe_decode_groups_static", L, bad, x, b) == 0
    torch.cuda.synchronize()
    assert torch.isnan(b["part"][3]).all() and torch.isfinite(b["part"][[0, 1, 2, 4]]).all()
    assert torch.isnan(b["y"]).all()
    assert _static_status(False) == ERR_ALIGN      # read without clearing: it stays
    assert _static_status(True) == ERR_ALIGN       # read and clear
    assert _static_status(False) == 0
    good = _bufs(22)
    assert _call("qmoe_decode_groups_static", L, c, x, good) == 0
    torch.cuda.synchronize()
    assert torch.isfinite(good["y"]).all() and _static_status(False) == 0


def test_static_entry_point_rejects_k_over_limit(layer):
    import _qmoe_lib as C
    c = _case(layer, 22)
    c["K"] = 97   # QMOE_STATIC_MAX_K + 1: refused before any work (QMOE_ERR_SCRATCH_LIMIT)
    assert _call("qmoe_decode_groups_static", layer, c, layer["xs"][0], _bufs(97)) == 9
    assert "static scratch" in C.status_string(9)
