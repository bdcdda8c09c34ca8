"""CPU-only checks of the boundary: the library builds for sm_100a, loads, exports every function the
header declares, the ctypes signature table covers the header exactly, and argument validation
rejects bad calls before any CUDA work (no GPU needed for those paths)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qmoe_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"^[A-Za-z_][\w \*]*?\b((?:qmoe|dq)_\w+)\s*\(", src, flags=re.M))


@pytest.fixture(scope="module")
def L():
    import _qmoe_lib
    if not os.path.exists(_qmoe_lib.LIB_PATH):
        import qmoe_build
        qmoe_build.build()
    return _qmoe_lib


def test_header_parse():
    names = declared()
    assert "qmoe_decode_groups" in names and "dq_gemv_fp8" in names
    assert len(names) >= 15


def test_every_declared_symbol_exported(L):
    lib = ctypes.CDLL(L.LIB_PATH)
    for name in sorted(declared()):
        assert hasattr(lib, name), name


def test_signature_table_matches_header(L):
    assert set(L.SIGNATURES) == declared()


def test_version_and_status_strings(L):
    assert "sm_100a" in L.version()
    assert L.status_string(0) == "ok"
    assert L.status_string(4) == "device-side wait timed out"


def test_null_and_shape_checks_need_no_gpu(L):
    lib = L.lib()
    assert lib.qmoe_decode_up(None, 0, 0, None, 22, None, None, 1, None, None) == 5       # NULL
    fake = ctypes.c_void_p(16)
    assert lib.qmoe_decode_up(fake, 1548288, 1, fake, 0, fake, fake, 1, fake, None) == 1  # K = 0
    assert lib.qmoe_decode_up(fake, 1548290, 1, fake, 22, fake, fake, 1, fake, None) == 2  # stride not 16-aligned
    assert lib.qmoe_decode_up(fake, 1548288, 1, fake, 22, fake, fake, 9, fake, None) == 6  # dtype
    assert lib.dq_gemv_fp8(fake, fake, fake, 1, 5, 16, 64, fake, None) == 1                 # M > 4
    assert lib.dq_gemv_nvfp4(fake, fake, fake, fake, 1, 1, 16, 48, fake, None) == 1         # K % 32
    assert lib.qmoe_decode_groups_workspace_bytes(22) >= 256 + 22 * 168 * 2
    assert lib.qmoe_decode_groups_workspace_bytes(0) == 0


def test_no_gpu_means_device_error(L):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = L.lib()
    fake = ctypes.c_void_p(16)
    # valid arguments, no CUDA device: the device check refuses (no fallback path exists)
    assert lib.qmoe_decode_up(fake, 1548288, 1, fake, 22, fake, fake, 1, fake, None) == 7
    assert lib.qmoe_copy_async(fake, fake, 64, None) == 7
    assert lib.qmoe_set_wait_cycles(300) == 7


def test_route_decode_argument_checks_need_no_gpu(L):
    lib = L.lib()
    f = ctypes.c_void_p(16)
    args = lambda ne, k: (f, f, ne, k, 5.0, 0, f, 3096576, f, f, f, f, f, f, None)
    assert lib.qmoe_route_decode(None, *args(512, 22)[1:]) == 5      # QMOE_ERR_NULL
    assert lib.qmoe_route_decode(*args(512, 33)) == 1                # top_k > 32
    assert lib.qmoe_route_decode(*args(1025, 22)) == 1               # n_experts > 1024
    assert lib.qmoe_route_decode(*args(16, 22)) == 1                 # top_k > n_experts


def test_copy_async_argument_checks_need_no_gpu(L):
    lib = L.lib()
    fake = ctypes.c_void_p(16)
    assert lib.qmoe_copy_async(None, None, 0, None) == 0     # nothing to copy: no CUDA call at all
    assert lib.qmoe_copy_async(None, fake, 8, None) == 5     # QMOE_ERR_NULL
    assert lib.qmoe_copy_async(fake, None, 8, None) == 5


def test_python_mirror_refuses_cpu_tensors(L):
    import torch
    import qmoe_ns
    blk = torch.zeros(1, qmoe_ns.BLOCK, dtype=torch.uint8)
    with pytest.raises(L.QmoeError):
        qmoe_ns.from_T_fast(blk, torch.zeros(qmoe_ns.LAT * qmoe_ns.KB_DN, dtype=torch.uint8))


def test_prefill_and_ep_argument_checks_need_no_gpu(L):
    """qmoe_prefill_grouped / qmoe_ep_* refuse bad arguments before touching a device, with the documented
    codes; with valid arguments and no GPU the device check refuses (no CPU fallback)."""
    import torch
    lib = L.lib()
    fake = ctypes.c_void_p(4096)          # 256-byte aligned stand-in pointer (never dereferenced)
    BLK = 3096576
    T, K, NE = 8, 22, 512
    need = lib.qmoe_prefill_workspace_bytes(T, K, NE, 0)
    assert need > 0
    assert lib.qmoe_prefill_workspace_bytes(0, K, NE, 0) == 0                # T out of range
    assert lib.qmoe_prefill_workspace_bytes(T, 33, NE, 0) == 0               # topk > 32
    assert lib.qmoe_prefill_workspace_bytes(2 * T, K, NE, 0) > need         # grows with T
    need_t = lib.qmoe_prefill_workspace_bytes(T, K, NE, 1)
    # a T-layout store adds one converted down half (1,548,288 B) per expert the prompt can use: min(NE, T*K)
    assert need_t - need == min(NE, T * K) * 1548288

    def pf(store=fake, stride=BLK, ne=NE, lt=1, ids=fake, w=fake, s2=fake, x=fake, dt=1, t=T, k=K, out=fake,
           ws=fake, wsb=need_t):
        return lib.qmoe_prefill_grouped(store, stride, ne, lt, ids, w, s2, x, dt, t, k, out, ws, wsb, None)

    assert pf(store=None) == 5
    assert pf(ws=None) == 5
    assert pf(t=0) == 1
    assert pf(k=33) == 1
    assert pf(ne=1025) == 1
    assert pf(stride=BLK - 16) == 1                                      # stride below one block
    assert pf(dt=9) == 6
    assert pf(stride=BLK + 8) == 2                                       # stride not a multiple of 16
    assert pf(x=ctypes.c_void_p(4096 + 8)) == 2                          # activations not 16-byte aligned
    assert pf(ws=ctypes.c_void_p(4096 + 16)) == 2                        # workspace not 256-byte aligned
    assert pf(wsb=need_t - 1) == 8                                       # workspace too small
    assert pf(lt=0, wsb=need) != 8                                       # the orig layout needs no conversion area
    if not torch.cuda.is_available():
        assert pf() == 7

    def pack(x=fake, ids=fake, w=fake, t=T, k=K, ne=NE, world=8, sx=fake, sm=fake, row=fake, cnt=fake):
        return lib.qmoe_ep_dispatch_pack(x, 1, ids, w, t, k, ne, world, sx, sm, row, cnt, None)

    assert pack(x=None) == 5
    assert pack(world=0) == 1
    assert pack(ne=511) == 1                                             # experts do not split over 8 ranks
    assert pack(sx=ctypes.c_void_p(4096 + 4)) == 2
    assert lib.qmoe_ep_combine(None, fake, T, 8, fake, None) == 5
    assert lib.qmoe_ep_combine(fake, fake, 0, 8, fake, None) == 1
    if not torch.cuda.is_available():
        assert pack() == 7
        assert lib.qmoe_ep_combine(fake, fake, T, 8, fake, None) == 7
