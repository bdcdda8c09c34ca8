"""Drop-in replacement of the reference's `dense_q` module (helgard-orlm/nemotron-super-8gb dense_q.py):
the dense part of Nemotron kept in its checkpoint formats (FP8 e4m3 per-tensor scale; NVFP4 = e2m1 +
e4m3 per 16 + weight_scale_2), multiplied by libqmoe_b200's sm_100a GEMV kernels.

Same quantized-weight dict {"fmt", "w", "sc", "s", "N", "K"} (dense_q.py:237-247), same functions.
Dispatch (dense_q.py:215-234): M == 1 -> gemv; 2 <= M <= MB_MAX -> gemv_mb (weights read once for all
vectors; the reference's limit is 2, these kernels take up to 4); larger M -> exact dequantization to
bf16 in row chunks (dq_dequant_rows) + F.linear (cuBLAS), as the reference does.
"""
import types

import torch
import torch.nn.functional as F

import _qmoe_lib as C

SCR_MIB = 64
_SCR = {}
MB_ON = True
MB_MAX = 4
# Kept for API compatibility (dense_q.py:156-164); the CUDA kernels choose their own launch shapes.
CFG = {"fp8": dict(BLOCK_N=16, BK=256, NSPLIT=1, num_warps=4), "nvfp4": dict(BLOCK_N=16, GB=8, NSPLIT=1, num_warps=2)}
CFG_BY_SHAPE = {}
E2M1_T = None


def _gemv(q, x2, M):
    N, K = q["N"], q["K"]
    x2 = x2.contiguous()
    out = torch.empty(M, N, dtype=torch.float32, device=x2.device)
    st = C.stream_of(x2)
    if q["fmt"] == "fp8":
        C.call("dq_gemv_fp8", C.ptr(q["w"]), C.ptr(q["s"]), C.ptr(x2), C.dtype_code(x2), M, N, K, C.ptr(out), st)
    else:
        C.call("dq_gemv_nvfp4", C.ptr(q["w"]), C.ptr(q["sc"]), C.ptr(q["s"]), C.ptr(x2), C.dtype_code(x2), M, N, K,
               C.ptr(out), st)
    return out


def gemv(q, x):
    """dense_q.py:199-212: x [K] (any float) -> y float32 [N]."""
    return _gemv(q, x.reshape(1, -1), 1)[0]


def gemv_mb(q, x):
    """dense_q.py:139-152: x [M,K], M <= MB_MAX -> y float32 [M,N]; the weight is read once."""
    M = x.shape[0]
    assert M <= MB_MAX
    return _gemv(q, x, M)


def _lut(dev):
    """dense_q.py:170-176 (kept for callers that use the table directly)."""
    global E2M1_T
    if E2M1_T is None or E2M1_T.device != torch.device(dev):
        v = torch.tensor([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], dtype=torch.float32,
                         device=dev)
        a = torch.arange(256, device=dev)
        E2M1_T = torch.stack([v[a & 15], v[a >> 4]], -1)
    return E2M1_T


def dequant_rows(q, r0, r1, out):
    """dense_q.py:179-188: rows [r0, r1) -> out [r1-r0, K] (bf16, fp16 or fp32), bit-exact."""
    if not out.is_contiguous():
        raise C.QmoeError("out must be contiguous")
    sc = q.get("sc")
    C.call("dq_dequant_rows", 0 if q["fmt"] == "fp8" else 1, C.ptr(q["w"]), C.ptr(sc) if sc is not None else None,
           C.ptr(q["s"]), q["N"], q["K"], r0, r1, C.ptr(out), C.dtype_code(out), C.stream_of(out))
    return out


def dequant(q):
    """dense_q.py:191-196: whole weight -> bf16 [N, K]."""
    out = torch.empty(q["N"], q["K"], dtype=torch.bfloat16, device=q["w"].device)
    return dequant_rows(q, 0, q["N"], out)


def qlinear(q, x):
    """dense_q.py:215-234: like F.linear(x, W_bf16) without bias: [..., K] -> [..., N] in x.dtype."""
    sh = x.shape
    x2 = x.reshape(-1, sh[-1])
    M, N = x2.shape[0], q["N"]
    if M == 1:
        return gemv(q, x2[0]).to(x.dtype).view(*sh[:-1], N)
    if M <= MB_MAX and MB_ON:
        return gemv_mb(q, x2).to(x.dtype).view(*sh[:-1], N)
    dev = x.device
    rows = max(1, min(N, SCR_MIB * 2**20 // (2 * q["K"])))
    scr = _SCR.get(dev)
    if scr is None or scr.numel() < rows * q["K"]:
        scr = _SCR[dev] = torch.empty(SCR_MIB * 2**20 // 2, dtype=torch.bfloat16, device=dev)
    y = torch.empty(M, N, dtype=x.dtype, device=dev)
    for r in range(0, N, rows):
        r1 = min(r + rows, N)
        w = dequant_rows(q, r, r1, scr[:(r1 - r) * q["K"]].view(r1 - r, q["K"]))
        y[:, r:r1] = F.linear(x2, w.to(x.dtype) if x.dtype != torch.bfloat16 else w)
    return y.view(*sh[:-1], N)


def load_q(ck, base, dev):
    """dense_q.py:237-247: checkpoint tensors under `base` -> quantized dict on `dev`, or None."""
    w = ck.get(base + ".weight")
    if base + ".weight_scale_2" in ck:
        sc = ck.get(base + ".weight_scale")
        return {"fmt": "nvfp4", "w": w.to(dev), "sc": sc.view(torch.uint8).to(dev),
                "s": ck.get(base + ".weight_scale_2").float().reshape(1).to(dev), "N": w.shape[0], "K": w.shape[1] * 2}
    if base + ".weight_scale" in ck and w.dtype == torch.float8_e4m3fn:
        return {"fmt": "fp8", "w": w.view(torch.uint8).to(dev),
                "s": ck.get(base + ".weight_scale").float().reshape(1).to(dev), "N": w.shape[0], "K": w.shape[1]}
    return None


def _fwd(self, x):
    return qlinear(self._q, x)


def attach(lin, q):
    """dense_q.py:254-261: nn.Linear -> quantized: the bf16 weight is released, forward goes to qlinear,
    .weight becomes the quantized bytes on the device."""
    assert lin.bias is None
    lin._parameters.pop("weight", None)
    lin._q = q
    object.__setattr__(lin, "weight", q["w"])
    lin.forward = types.MethodType(_fwd, lin)


def nbytes(q):
    return sum(t.numel() * t.element_size() for k, t in q.items() if isinstance(t, torch.Tensor))
