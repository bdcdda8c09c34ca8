"""GPU parity of the HBM-resident store and the drop-in experts module (nemotron-super-8gb_b200/expert_store.py)
on engine files in the reference's format (repack.py:1-7), written from synthetic NVFP4 experts (config 0
recipe) in a small geometry of 2 MoE layers x 24 experts:
* the loaded store is byte-identical to the file, in the file's layout and after conversion on the device
  (orig -> T equals qmoe_to_T of each block; a T-layout file loads as written);
* RoutedExperts.forward matches the fp64 oracle within BF16_TOL (rel-L2) for one token (decode kernels,
  both layouts) and for a prompt (grouped prefill GEMM, both layouts), returning hidden_states.dtype."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
NL, NE, K = 2, 24, 22
BF16_TOL = 2.0 ** -8


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def engine(tmp_path_factory):
    import expert_store as ES
    import qmoe_synth as S
    g = S.seeded(71, DEV)
    m_hat = S.unit_dir(g, DEV)
    blk, s2, _ = S.expert_blocks(NL * NE, 0.075, m_hat, g, DEV)
    scal = np.zeros((NL, NE, 4), np.float32)
    scal[:, :, :2] = s2.float().cpu().numpy().reshape(NL, NE, 2)
    X = S.tokens(9, m_hat, g, DEV)
    d_orig = str(tmp_path_factory.mktemp("orig"))
    ES.write_engine_files(d_orig, blk, scal, layout="orig")
    import qmoe_ns as Q
    blkT = blk.clone()
    Q.to_T_batch(blkT)
    torch.cuda.synchronize()
    d_T = str(tmp_path_factory.mktemp("T"))
    ES.write_engine_files(d_T, blkT, scal, layout="T")
    return dict(d_orig=d_orig, d_T=d_T, blk=blk.cpu().numpy(), blkT=blkT.cpu().numpy(), scal=scal, X=X)


def test_store_bytes_and_conversion(engine):
    import expert_store as ES
    e = engine
    st = ES.ExpertStore(e["d_orig"], device=DEV, n_layers=NL, n_experts=NE, chunk_blocks=5, threads=3)
    assert st.layout == "orig"
    assert np.array_equal(st.blocks.cpu().numpy(), e["blk"])
    assert np.array_equal(st.s2.cpu().numpy(), e["scal"][:, :, :2])
    stT = ES.ExpertStore(e["d_orig"], device=DEV, n_layers=NL, n_experts=NE, layout="T", chunk_blocks=7)
    assert stT.layout == "T"
    assert np.array_equal(stT.blocks.cpu().numpy(), e["blkT"])
    fT = ES.ExpertStore(e["d_T"], device=DEV, n_layers=NL, n_experts=NE)
    assert fT.layout == "T"
    assert np.array_equal(fT.blocks.cpu().numpy(), e["blkT"])
    back = ES.ExpertStore(e["d_T"], device=DEV, n_layers=NL, n_experts=NE, layout="orig", shard=(4, 16))
    assert np.array_equal(back.layer(1).cpu().numpy(), e["blk"][NE + 4:NE + 16])


@pytest.mark.parametrize("layout", ["orig", "T"])
def test_routed_experts_decode_and_prompt(engine, layout):
    import expert_store as ES
    e = engine
    st = ES.ExpertStore(e["d_orig"], device=DEV, n_layers=NL, n_experts=NE, layout=layout)
    m = 1
    mod = ES.RoutedExperts(m, st)
    rng = np.random.default_rng(8 + (layout == "T"))
    X = e["X"]
    blocks = [e["blk"][m * NE + j] for j in range(NE)]
    s2m = e["scal"][m, :, :2]
    Xf = X.float().cpu().numpy()
    # one token: decode kernels
    ids = rng.permutation(NE)[:K].astype(np.int64)[None]
    w = rng.uniform(0.1, 1.0, (1, K)).astype(np.float32)
    y = mod(X[:1], torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV))
    assert y.shape == (1, 1024) and y.dtype == X.dtype
    ref, _, _ = O.moe_decode([blocks[j] for j in ids[0]], s2m[ids[0]], w[0], Xf[0])
    assert rel_l2(y.float().cpu().numpy()[0], ref) < BF16_TOL
    # a prompt: grouped prefill GEMM
    T = X.shape[0]
    ids = np.stack([rng.permutation(NE)[:K] for _ in range(T)]).astype(np.int64)
    w = rng.uniform(0.1, 1.0, (T, K)).astype(np.float32)
    y = mod(X, torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV))
    assert y.shape == (T, 1024) and y.dtype == X.dtype
    ref = O.prefill(blocks, s2m, ids.astype(np.int32), w, Xf)
    yn = y.float().cpu().numpy()
    assert rel_l2(yn, ref) < BF16_TOL
    assert max(rel_l2(yn[t], ref[t]) for t in range(T)) < BF16_TOL
