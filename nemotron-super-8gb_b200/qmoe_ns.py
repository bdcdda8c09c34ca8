"""Drop-in replacement of the reference's `qmoe_ns` module (helgard-orlm/nemotron-super-8gb qmoe_ns.py):
the NVFP4 routed experts of Nemotron-3.5-Super (latent 1024 -> 2688 -> 1024, ReLU^2, no gate), with
every function computed by libqmoe_b200 (hand-written sm_100a CUDA) through its C ABI.

Same names, argument order, buffer roles and return values as the reference; tensors must be CUDA
tensors, and calls launch asynchronously on torch's current stream. Activations are not quantized
(W4A16) in the decode and pair kernels: codes and block scales are decoded exactly, products are exact and
every sum is fp32, as in the reference's kernels (qmoe_ns.py:4). moe_prefill's tensor-core GEMMs take the
activations as three NVFP4 residual planes (rel-L2 about 5e-4 of the fp32 path, inside bf16 tolerance).
"""
import torch

import _qmoe_lib as C

LAT, INTER = 1024, 2688
BLOCK = 3096576
O_UW, O_US, O_DW, O_DS = 0, 1376256, 1548288, 2924544
KB_UP, G_UP = LAT // 2, LAT // 16
KB_DN, G_DN = INTER // 2, INTER // 16
assert O_DS + LAT * G_DN == BLOCK
UPB = O_DW
O_TW, O_TS = O_DW, O_DW + INTER * 512

# Kept for API compatibility (qmoe_ns.py:206, :242, :315). The CUDA kernels pick their own launch
# shapes; a `cfg` passed to the decode functions is accepted and ignored.
LIVE_CFG = dict(BR=256, NB=8, KS=8, num_warps=4)
GROUP_CFG = dict(BR=1024, KS=2, num_warps=2)
PAIRS_T_BR = 64

# qmoe_ns.py:391-392
E2M1 = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=torch.float32)
SWAP = False   # negative control: the high nibble taken as the even element (deliberately wrong)

_WS = {}


def _slots_args(slots):
    if slots.dtype != torch.uint8 or slots.dim() != 2 or slots.stride(1) != 1:
        raise C.QmoeError("slots must be a uint8 [S, bytes] tensor with contiguous rows")
    return C.ptr(slots), int(slots.stride(0)), int(slots.shape[0])


def _f32(t):
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise C.QmoeError("expected a contiguous float32 tensor")
    return C.ptr(t)


def _i32(t):
    if t.dtype != torch.int32 or not t.is_contiguous():
        raise C.QmoeError("expected a contiguous int32 tensor")
    return C.ptr(t)


def _act(x):
    x = x.contiguous()
    return x, C.ptr(x), C.dtype_code(x)


def moe_decode(slots_u8, sidx, s2, coef, x, h_buf, out_buf):
    """qmoe_ns.py:70-76. slots_u8 [S, BLOCK] u8 (orig layout) · sidx [K] int32 · s2 [K,2] f32 ·
    coef [K] f32 · x [1024] -> fp32 [1024] (the sum over K in slot order). Fills h_buf[:K], out_buf[:K]."""
    K = sidx.shape[0]
    sp, sb, ns = _slots_args(slots_u8)
    x, xp, xd = _act(x)
    y = torch.empty(LAT, dtype=torch.float32, device=x.device)
    C.call("qmoe_decode", sp, sb, ns, _i32(sidx), _f32(s2), _f32(coef), xp, xd, K, _f32(h_buf), _f32(out_buf),
           C.ptr(y), C.stream_of(x))
    return y


def moe_pairs(slots_u8, pslot, ptok, s2p, coefp, X, h_buf, out_buf):
    """qmoe_ns.py:127-133. P pairs (slot, token) -> out_buf[:P] fp32 [P,1024]; X [T,1024] contiguous;
    pslot/ptok int32 [P]; s2p [P,2] f32; coefp [P] f32. Fills h_buf[:P]."""
    P = pslot.shape[0]
    sp, sb, ns = _slots_args(slots_u8)
    X, xp, xd = _act(X)
    if P:
        C.call("qmoe_pairs", sp, sb, ns, _i32(pslot), _i32(ptok), _f32(s2p), _f32(coefp), xp, xd, X.shape[0], P,
               _f32(h_buf), _f32(out_buf), C.stream_of(X))
    return out_buf[:P]


def _workspace(dev, K):
    """Per (device, stream) workspace of qmoe_decode_groups, created zeroed and kept."""
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    need = int(C.lib().qmoe_decode_groups_workspace_bytes(K))
    ws = _WS.get(key)
    if ws is None or ws.numel() < need:
        ws = _WS[key] = torch.zeros(max(need, 1 << 16), dtype=torch.uint8, device=dev)
    return ws


def moe_decode_groups(slots_up, sidx, tab, s2, coef, x, h_buf, part_buf, gidx_buf, gcnt_buf, cfg=None):
    """qmoe_ns.py:245-255: up from slots_up (UPB or BLOCK row stride), live-group compaction, down over
    the live 16-neuron groups of the T-layout blocks at tab [K] int64 (device addresses), fixed-order sum.
    Leaves h_buf[:K], gidx_buf[:K], gcnt_buf[:K] as the reference does; part_buf[0,:K] holds the
    per-expert outputs coef_j * s2d_j * D_j h_j. Returns fp32 [1024]."""
    K = sidx.shape[0]
    sp, sb, ns = _slots_args(slots_up)
    x, xp, xd = _act(x)
    if tab.dtype != torch.int64 or not tab.is_cuda:
        raise C.QmoeError("tab must be a CUDA int64 tensor of block addresses")
    ws = _workspace(x.device, K)
    y = torch.empty(LAT, dtype=torch.float32, device=x.device)
    C.call("qmoe_decode_groups", sp, sb, ns, _i32(sidx), C.ptr(tab.contiguous()), _f32(s2), _f32(coef), xp, xd, K,
           _f32(h_buf), _i32(gidx_buf), _i32(gcnt_buf), _f32(part_buf), C.ptr(y), C.ptr(ws), ws.numel(),
           C.stream_of(x))
    return y


def decode_groups_status(device=None, clear=True):
    """Device-side status of the decode workspace on the current stream (synchronises it)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    ws = _WS.get((dev.index, torch.cuda.current_stream(dev).cuda_stream))
    if ws is None:
        return 0
    return int(C.lib().qmoe_workspace_status(C.ptr(ws), int(clear), C.stream_of(ws)))


def _live_lists(h_buf, K, idx_buf, cnt_buf):
    # the reference's torch glue (qmoe_ns.py:265-267), on the device
    live = h_buf[:K] > 0
    torch.sum(live, dim=1, dtype=torch.int32, out=cnt_buf[:K])
    idx_buf[:K] = torch.sort(live.to(torch.uint8), dim=1, descending=True, stable=True).indices.to(torch.int32)


def moe_decode_live2(slots_up, sidx, tab, s2, coef, x, h_buf, part_buf, idx_buf, cnt_buf, cfg=None):
    """qmoe_ns.py:260-271 (superseded by moe_decode_groups; same math). part_buf is scratch;
    idx_buf/cnt_buf receive the live-neuron lists as the reference leaves them."""
    K = sidx.shape[0]
    gidx = torch.empty(K, G_DN, dtype=torch.int32, device=x.device)
    gcnt = torch.empty(K, dtype=torch.int32, device=x.device)
    y = moe_decode_groups(slots_up, sidx, tab, s2, coef, x, h_buf, part_buf, gidx, gcnt)
    _live_lists(h_buf, K, idx_buf, cnt_buf)
    return y


def moe_decode_live(slots_up, sidx, tab, s2, coef, x, h_buf, out_buf, idx_buf, cnt_buf, BR=256, NB=8):
    """qmoe_ns.py:274-283 (superseded; same math). out_buf is scratch."""
    K = sidx.shape[0]
    part = out_buf[:K].view(1, K, LAT)
    return moe_decode_live2(slots_up, sidx, tab, s2, coef, x, h_buf, part, idx_buf, cnt_buf)


_PWS = {}


def _prefill_workspace(dev, T, topk, ne, layout_T):
    """Per (device, stream) workspace of qmoe_prefill_grouped, grown on demand; status word zeroed."""
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    need = int(C.lib().qmoe_prefill_workspace_bytes(T, topk, ne, int(bool(layout_T))))
    if need == 0:
        raise C.QmoeError(f"prefill shape out of range: T={T} topk={topk} n_experts={ne}")
    ws = _PWS.get(key)
    if ws is None or ws.numel() < need:
        _PWS.pop(key, None)
        ws = torch.empty(need + (need >> 3), dtype=torch.uint8, device=dev)
        ws[:256].zero_()
        _PWS[key] = ws
    return ws


def moe_prefill(store, ids, weights, s2, X, layout_T=True, out=None):
    """Prompt-path routed-expert forward (nem_super.py:295-348 as one call): X [T,1024], ids [T,topk]
    expert ids into store [E, >= BLOCK] u8 (one block per row), weights [T,topk], s2 [E,2] f32 ->
    fp32 [T,1024] = sum over k, in k order, of weights[t,k] * expert_{ids[t,k]}(X[t]).
    One expert-grouped, block-scaled NVFP4 GEMM per half on the tensor cores (activations as three NVFP4
    residual planes); layout_T: the down halves are in the T layout (those of the experts the prompt uses are
    converted to the orig layout inside the call; the result equals the orig-layout call's). Ids of -1 are
    skipped; the workspace is kept per (device, stream)."""
    if store.dtype != torch.uint8 or store.dim() != 2 or store.stride(1) != 1 or store.shape[1] < BLOCK:
        raise C.QmoeError("store must be a uint8 [E, >= BLOCK] tensor with contiguous rows")
    T, topk = ids.shape
    X, xp, xd = _act(X)
    if X.shape != (T, LAT):
        raise C.QmoeError("X must be [T, 1024] with T = ids.shape[0]")
    ids32 = ids.to(torch.int32).contiguous()
    w32 = weights.to(torch.float32).contiguous()
    s2c = s2.to(torch.float32).contiguous()
    if out is None:
        out = torch.empty(T, LAT, dtype=torch.float32, device=X.device)
    ws = _prefill_workspace(X.device, T, topk, store.shape[0], layout_T)
    C.call("qmoe_prefill_grouped", C.ptr(store), int(store.stride(0)), int(store.shape[0]), int(bool(layout_T)),
           C.ptr(ids32), C.ptr(w32), C.ptr(s2c), xp, xd, T, topk, _f32(out), C.ptr(ws), ws.numel(),
           C.stream_of(X))
    return out


def prefill_status(device=None, clear=True):
    """Device-side status of the prefill workspace on the current stream (synchronises it)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    ws = _PWS.get((dev.index, torch.cuda.current_stream(dev).cuda_stream))
    if ws is None:
        return 0
    return int(C.lib().qmoe_workspace_status(C.ptr(ws), int(clear), C.stream_of(ws)))


def set_wait_cycles(cycles, device=None):
    """Bound, in SM clock cycles, on each device-side wait of moe_prefill's GEMM pipelines on the device (the
    current one by default), from the next call on; cycles <= 0 restores the default (4e9, about 2 s). A wait
    that runs out records QMOE_ERR_TIMEOUT (prefill_status() == 4) and the kernel stops after its copies and
    MMAs in flight complete. No counterpart in the reference."""
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        C.call("qmoe_set_wait_cycles", int(cycles))


def moe_pairs_T(slots_u8, pslot, ptok, s2p, coefp, X, h_buf, out_buf):
    """qmoe_ns.py:318-324: pairs over T-layout slots. The slots used are converted to the orig layout
    in a scratch copy (from_T) and the pairs kernels run on it, as the reference engine's prompt path
    does (nem_super.py:324-339). The distinct slots are found on the device with a fixed bound of
    min(P, S) rows (a sort, a first-occurrence scan and a scatter), so nothing waits for the host; rows past
    the distinct count repeat the smallest slot and are converted but never read."""
    P = pslot.shape[0]
    if P == 0:
        return out_buf[:0]
    n = min(P, slots_u8.shape[0])
    srt, order = torch.sort(pslot.long())
    first = torch.ones_like(srt, dtype=torch.bool)
    first[1:] = srt[1:] != srt[:-1]
    rank = torch.cumsum(first, 0) - 1                    # index of each sorted pair's slot among the distinct ones
    uniq = srt[:1].expand(n).clone()
    uniq.scatter_(0, rank, srt)                          # equal ranks write equal slots
    inv = torch.empty_like(rank).scatter_(0, order, rank)
    tmp = slots_u8.index_select(0, uniq).contiguous()
    from_T_batch(tmp)
    return moe_pairs(tmp, inv.to(torch.int32).contiguous(), ptok, s2p, coefp, X, h_buf, out_buf)


def from_T_fast(blks, scratch):
    """qmoe_ns.py:345-353: [N, BLOCK] on the device, T -> orig in place; scratch u8 >= N*1376256."""
    N = blks.shape[0]
    if blks.dtype != torch.uint8 or blks.stride(0) != BLOCK or blks.stride(1) != 1:
        raise C.QmoeError("blks must be uint8 [N, BLOCK] with contiguous rows")
    if scratch.numel() < N * LAT * KB_DN:
        raise C.QmoeError("scratch too small")
    C.call("qmoe_from_T", C.ptr(blks), N, C.ptr(scratch), C.stream_of(blks))
    return blks


def _scratch(blks):
    return torch.empty(max(1, blks.shape[0]) * LAT * KB_DN, dtype=torch.uint8, device=blks.device)


def from_T_batch(blks):
    """qmoe_ns.py:378-387: [N, BLOCK] on the device, T -> orig in place."""
    return from_T_fast(blks, _scratch(blks))


def to_T_batch(blks):
    """repack_T.py:27-35: [N, BLOCK] on the device, orig -> T in place."""
    N = blks.shape[0]
    if blks.dtype != torch.uint8 or blks.stride(0) != BLOCK or blks.stride(1) != 1:
        raise C.QmoeError("blks must be uint8 [N, BLOCK] with contiguous rows")
    C.call("qmoe_to_T", C.ptr(blks), N, C.ptr(_scratch(blks)), C.stream_of(blks))
    return blks


def to_T(blk):
    """qmoe_ns.py:356-364: orig-layout block (u8 [BLOCK], on the device) -> T layout (new tensor)."""
    out = blk.clone().view(1, BLOCK)
    return to_T_batch(out).view(BLOCK)


def from_T(blk):
    """qmoe_ns.py:367-375: T-layout block -> orig layout (new tensor)."""
    out = blk.clone().view(1, BLOCK)
    return from_T_batch(out).view(BLOCK)


def deq(w_u8, s_e4m3_u8, ws2):
    """qmoe_ns.py:395-404: w_u8 [N, K/2] · s [N, K/16] (e4m3 bytes) · ws2 -> fp32 [N, K], bit-exact."""
    w = w_u8.contiguous()
    if SWAP:
        w = ((w >> 4) | (w << 4)).contiguous()
    s = s_e4m3_u8.contiguous()
    N, K = w.shape[0], w.shape[1] * 2
    out = torch.empty(N, K, dtype=torch.float32, device=w.device)
    C.call("qmoe_deq", C.ptr(w), C.ptr(s), float(ws2), N, K, C.ptr(out), C.stream_of(w))
    return out


def block_deq(blk_u8, s2):
    """qmoe_ns.py:407-412: block (u8 [BLOCK], orig layout) -> up [2688,1024], down [1024,2688] fp32."""
    b = blk_u8
    u = deq(b[O_UW:O_US].view(INTER, KB_UP), b[O_US:O_DW].view(INTER, G_UP), float(s2[0]))
    d = deq(b[O_DW:O_DS].view(LAT, KB_DN), b[O_DS:BLOCK].view(LAT, G_DN), float(s2[1]))
    return u, d
