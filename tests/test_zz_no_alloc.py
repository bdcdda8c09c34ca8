"""qmoe_decode_groups_static — the decode-step layer for callers that cannot allocate device memory (hosts
whose HBM is already committed to their own pool, code inside a CUDA graph capture that refuses
allocation calls, foreign-language hosts that only pass pointers through). It keeps its scratch in a
static device array inside the library instead of a caller workspace.

Checked here through the C ABI against the workspace entry point qmoe_decode_groups on the same inputs,
on two calls in a row (the second call finds the first call's leftovers in the shared array), plus the
size limit. The file name sorts last so that a run stopping at the first failure has run every other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

BF16_TOL = 2.0 ** -8
DEV = "cuda"


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
    K = 22
    blk, s2, _ = S.expert_blocks(K, 0.075, m_hat, g, DEV)
    Q.to_T_batch(blk)
    xs = S.tokens(2, m_hat, g, DEV)
    coef = (torch.rand(K, generator=g, device=DEV) * 5).float()
    tab = torch.tensor([blk[j].data_ptr() for j in range(K)], dtype=torch.int64, device=DEV)
    sidx = torch.arange(K, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    return dict(blk=blk, s2=s2.float().contiguous(), xs=xs, coef=coef, tab=tab, sidx=sidx, K=K)


def _bufs(K):
    return dict(h=torch.empty(K, 2688, device=DEV), part=torch.empty(K, 1024, device=DEV),
                gidx=torch.empty(K, 168, dtype=torch.int32, device=DEV), gcnt=torch.empty(K, dtype=torch.int32, device=DEV),
                y=torch.empty(1024, device=DEV))


def _call(name, L, x, b, extra=()):
    import _qmoe_lib as C
    blk = L["blk"]
    args = [C.ptr(blk), blk.stride(0), blk.shape[0], C.ptr(L["sidx"]), C.ptr(L["tab"]), C.ptr(L["s2"]),
            C.ptr(L["coef"]), C.ptr(x), C.dtype_code(x), L["K"], C.ptr(b["h"]), C.ptr(b["gidx"]), C.ptr(b["gcnt"]),
            C.ptr(b["part"]), C.ptr(b["y"])]
    return getattr(C.lib(), name)(*args, *extra, C.stream_of(x))


def test_static_entry_point_matches_workspace_entry_point(layer):
    import _qmoe_lib as C
    L = layer
    K = L["K"]
    ws = torch.zeros(int(C.lib().qmoe_decode_groups_workspace_bytes(K)), dtype=torch.uint8, device=DEV)
    for call in range(2):   # two calls in a row, different tokens
        x = L["xs"][call]
        ref = _bufs(K)
        assert _call("qmoe_decode_groups", L, x, ref, (C.ptr(ws), ws.numel())) == 0
        got = _bufs(K)
        assert _call("qmoe_decode_groups_static", L, x, got) == 0
        torch.cuda.synchronize()
        assert rel_l2(got["y"].cpu().numpy(), ref["y"].cpu().numpy()) < BF16_TOL
        assert rel_l2(got["h"].cpu().numpy(), ref["h"].cpu().numpy()) < BF16_TOL
        assert torch.equal(got["gidx"], ref["gidx"]) and torch.equal(got["gcnt"], ref["gcnt"])
        assert torch.isfinite(got["y"]).all()


def test_static_entry_point_rejects_k_over_limit(layer):
    import _qmoe_lib as C
    L = dict(layer)
    K = 97   # QMOE_STATIC_MAX_K + 1: refused before any work (QMOE_ERR_SCRATCH_LIMIT)
    L["K"] = K
    assert _call("qmoe_decode_groups_static", L, layer["xs"][0], _bufs(K)) == 9
    assert "static scratch" in C.status_string(9)
