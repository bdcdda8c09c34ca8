"""Seeded input generators shared by tests/golden/make_golden.py (which runs the reference on them)
and the tests (which regenerate the same inputs and compare against the stored golden outputs).

numpy's PCG64 `default_rng(seed)` streams are stable across numpy versions, so the inputs need not
be stored: only the reference's outputs are (golden.npz / golden.json).
"""
import numpy as np

LAT, INTER = 1024, 2688
BLOCK = 3096576
O_UW, O_US, O_DW, O_DS = 0, 1376256, 1548288, 2924544

# e4m3 bytes 0x28..0x47: positive normal scales 2^-2 .. 2^1*1.875 (no NaN, no sign)
SC_LO, SC_HI = 0x28, 0x48


def rand_block(seed):
    """An orig-layout expert block (qmoe_ns.py:9-14 offsets) with uniform random nibbles and valid
    positive e4m3 block scales."""
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, BLOCK, dtype=np.uint8)
    blk[O_US:O_DW] = rng.integers(SC_LO, SC_HI, O_DW - O_US, dtype=np.uint8)
    blk[O_DS:BLOCK] = rng.integers(SC_LO, SC_HI, BLOCK - O_DS, dtype=np.uint8)
    return blk


def rand_bytes_block(seed):
    """Any bytes at all: for the pure byte permutations to_T / from_T."""
    return np.random.default_rng(seed).integers(0, 256, BLOCK, dtype=np.uint8)


def bf16_round(x):
    """float32 -> nearest-even bf16 value, returned as float32."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = 0x7FFF + ((u >> 16) & 1)
    return (((u + r) >> 16).astype(np.uint32) << 16).view(np.float32)


def decode_case(seed=100, K=4):
    """Inputs of the moe_decode golden case: K blocks, s2 [K,2], coef [K], x (bf16 values) [1024]."""
    rng = np.random.default_rng(seed)
    blocks = [rand_block(seed + 1 + j) for j in range(K)]
    s2 = rng.uniform(0.002, 0.02, (K, 2)).astype(np.float32)
    coef = rng.uniform(0.1, 1.0, K).astype(np.float32)
    x = bf16_round(rng.normal(0, 0.5, LAT).astype(np.float32))
    return blocks, s2, coef, x


def pairs_case(seed=200, NB=4, T=3, per_tok=2):
    """Inputs of the moe_pairs golden case: NB slot blocks, T tokens, each routed to `per_tok` slots."""
    rng = np.random.default_rng(seed)
    blocks = [rand_block(seed + 1 + j) for j in range(NB)]
    s2 = rng.uniform(0.002, 0.02, (NB, 2)).astype(np.float32)
    X = bf16_round(rng.normal(0, 0.5, (T, LAT)).astype(np.float32))
    sel = np.stack([rng.permutation(NB)[:per_tok] for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, (T, per_tok)).astype(np.float32)
    t_i = np.repeat(np.arange(T, dtype=np.int32), per_tok)
    k_i = np.tile(np.arange(per_tok, dtype=np.int32), T)
    pslot = sel[t_i, k_i].astype(np.int32)
    s2p = s2[pslot]
    coefp = w[t_i, k_i].astype(np.float32)
    return blocks, pslot, t_i, s2p, coefp, X


def dense_case(fmt, seed, N=32, K=256, M=2):
    """Quantized-weight dict fields (dense_q.py:237-247) with random bytes, plus x [M,K] bf16 values."""
    rng = np.random.default_rng(seed)
    if fmt == "fp8":
        w = rng.integers(0, 256, (N, K), dtype=np.uint8)
        w[(w & 0x7F) == 0x7F] = 0x10          # no NaN encodings
        sc = None
        s = np.float32(0.0173)
    else:
        w = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
        sc = rng.integers(SC_LO, SC_HI, (N, K // 16), dtype=np.uint8)
        s = np.float32(0.00731)
    x = bf16_round(rng.normal(0, 1.0, (M, K)).astype(np.float32))
    return w, sc, s, x


def route_case(seed=300, T=4, E=512, hidden=64):
    """Router inputs: hidden [T,hidden] fp32, gate weight [E,hidden], correction bias [E]."""
    rng = np.random.default_rng(seed)
    h = rng.normal(0, 1.0, (T, hidden)).astype(np.float32)
    w = rng.normal(0, 0.02, (E, hidden)).astype(np.float32)
    b = rng.normal(0, 0.01, E).astype(np.float32)
    return h, w, b
