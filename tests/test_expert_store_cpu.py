"""ExpertStore (nemotron-super-8gb_b200/expert_store.py) file handling on CPU: the reference's engine files
(repack.py:1-7: experts.bin with block m*512 + e, experts_scal.npy [L, E, 4], experts.layout) are read byte
for byte, layers and expert shards are selected as asked, and malformed or half-converted files are refused.
A small stand-in geometry (3 layers x 5 experts) keeps the files small."""
import os

import numpy as np
import pytest
import torch

import vectors as V

NL, NE = 3, 5


@pytest.fixture()
def engine(tmp_path):
    import expert_store as ES
    blocks = np.stack([V.rand_bytes_block(900 + i) for i in range(NL * NE)])
    scal = np.random.default_rng(5).uniform(0.001, 0.02, (NL, NE, 4)).astype(np.float32)
    ES.write_engine_files(str(tmp_path), blocks, scal, layout="orig")
    return str(tmp_path), blocks, scal


def test_load_all_bytes_and_scales(engine):
    import expert_store as ES
    d, blocks, scal = engine
    st = ES.ExpertStore(d, device="cpu", n_layers=NL, n_experts=NE, chunk_blocks=2, threads=2)
    assert st.layout == "orig" and st.e_local == NE
    assert np.array_equal(st.blocks.numpy(), blocks)
    assert np.array_equal(st.s2.numpy(), scal[:, :, :2])


def test_layers_and_shard(engine):
    import expert_store as ES
    d, blocks, scal = engine
    st = ES.ExpertStore(d, device="cpu", layers=[2, 0], shard=(1, 4), n_layers=NL, n_experts=NE, chunk_blocks=2)
    assert st.e_local == 3
    for i, m in enumerate([2, 0]):
        assert np.array_equal(st.layer(i).numpy(), blocks[m * NE + 1:m * NE + 4])
        assert np.array_equal(st.s2[i].numpy(), scal[m, 1:4, :2])
    assert st.index(0) == 1
    ids = torch.tensor([3, 1])
    assert st.slot_index(st.index(0), ids).tolist() == [3 + 2, 3 + 0]
    with pytest.raises(KeyError):
        st.index(1)


def test_layout_markers(engine, tmp_path):
    import _qmoe_lib as C
    import expert_store as ES
    d, _, _ = engine
    with open(os.path.join(d, "experts.layout"), "w") as f:
        f.write("T\n")
    assert ES.read_layout(d) == "T"
    st = ES.ExpertStore(d, device="cpu", n_layers=NL, n_experts=NE)
    assert st.layout == "T"
    open(os.path.join(d, "experts.layout.inprogress"), "w").close()
    with pytest.raises(C.QmoeError):
        ES.read_layout(d)
    os.remove(os.path.join(d, "experts.layout.inprogress"))
    with open(os.path.join(d, "experts.layout"), "w") as f:
        f.write("bogus\n")
    with pytest.raises(C.QmoeError):
        ES.read_layout(d)
    os.remove(os.path.join(d, "experts.layout"))
    assert ES.read_layout(d) == "orig"    # no marker: the orig layout (nem_super.py:92)


def test_refusals(engine):
    import _qmoe_lib as C
    import expert_store as ES
    d, blocks, scal = engine
    with pytest.raises(C.QmoeError):        # file shorter than the geometry
        ES.ExpertStore(d, device="cpu", n_layers=NL + 1, n_experts=NE)
    with pytest.raises(C.QmoeError):        # layout conversion needs the GPU
        ES.ExpertStore(d, device="cpu", n_layers=NL, n_experts=NE, layout="T")
    with pytest.raises(ValueError):
        ES.ExpertStore(d, device="cpu", n_layers=NL, n_experts=NE, shard=(3, 9))
    st = ES.ExpertStore(d, device="cpu", n_layers=NL, n_experts=NE, shard=(0, 2))
    with pytest.raises(ValueError):         # a shard cannot serve a whole layer
        ES.RoutedExperts(0, st)
