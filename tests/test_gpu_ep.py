"""GPU parity of the expert-parallel pieces (csrc/ep.cu through ep.CudaOps): the dispatch pack against the
oracle's restatement (bit-exact), and a whole expert-parallel layer with the all-to-all exchanges emulated
inside one process for 2 and 4 ranks, against the fp64 oracle layer and the single-GPU prefill. When the
box has two GPUs, the same layer also runs over NCCL with one process per GPU."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 2.0 ** -8
DEV = "cuda"
NE = 16


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def bank():
    import qmoe_ns as Q
    import qmoe_synth as S
    g = S.seeded(61, DEV)
    m_hat = S.unit_dir(g, DEV)
    blk, s2, _ = S.expert_blocks(NE, 0.075, m_hat, g, DEV)
    blkT = blk.clone()
    Q.to_T_batch(blkT)
    X = S.tokens(4 * 24, m_hat, g, DEV)
    torch.cuda.synchronize()
    return dict(blk=blk, blkT=blkT, s2=s2.float().contiguous(), X=X, blk_np=blk.cpu().numpy(),
                s2_np=s2.float().cpu().numpy())


def _route(T, k, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(NE)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, (T, k)).astype(np.float32)
    return ids, w


@pytest.mark.parametrize("world", [2, 4])
def test_ep_pack_bit_exact(bank, world):
    import ep
    T, k = 24, 6
    ids, w = _route(T, k, 5 + world)
    X = bank["X"][:T]
    sx, meta, row_of, cnt = ep.CudaOps().pack(X, torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV), NE, world)
    rx, ri, rw, rrow, rcnt = O.ep_pack(X.view(torch.int16).cpu().numpy(), ids, w, NE, world)
    assert np.array_equal(cnt.cpu().numpy(), rcnt)
    assert np.array_equal(row_of.cpu().numpy(), rrow)
    m = meta.cpu().numpy()
    assert np.array_equal(m[:, :, :k], ri)
    sxn = sx.view(torch.int16).cpu().numpy()
    for d in range(world):
        c = rcnt[d]
        assert np.array_equal(sxn[d, :c], rx[d, :c])
        assert np.array_equal(m[d, :c, k:].view(np.float32), rw[d, :c])


def _emulated_layer(bank, world, X_ranks, ids_ranks, w_ranks, layout_T=True):
    """All ranks of an expert-parallel layer in one process; all_to_all = block transpose."""
    import ep
    ops = ep.CudaOps()
    el = NE // world
    store = bank["blkT"] if layout_T else bank["blk"]
    packs = [ops.pack(X_ranks[r], ids_ranks[r], w_ranks[r], NE, world) for r in range(world)]
    T = X_ranks[0].shape[0]
    k = ids_ranks[0].shape[1]
    parts = []
    for r in range(world):   # rank r receives block r of every source
        rx = torch.stack([packs[s][0][r] for s in range(world)])
        rm = torch.stack([packs[s][1][r] for s in range(world)])
        part = ops.local(store[r * el:(r + 1) * el], bank["s2"][r * el:(r + 1) * el], rx.view(world * T, -1),
                         rm.view(world * T, 2 * k), layout_T)
        parts.append(part.view(world, T, -1))
    outs = []
    for s in range(world):   # source s gets back block s of every rank's partials
        rp = torch.stack([parts[r][s] for r in range(world)])
        outs.append(ops.combine(rp, packs[s][2]))
    return outs


@pytest.mark.parametrize("world,layout_T", [(2, True), (4, True), (2, False)])
def test_ep_layer_emulated(bank, world, layout_T):
    import qmoe_ns as Q
    T, k = 24, 6
    X_r, ids_r, w_r, ids_np, w_np = [], [], [], [], []
    for r in range(world):
        ids, w = _route(T, k, 40 + r)
        ids_np.append(ids)
        w_np.append(w)
        X_r.append(bank["X"][r * T:(r + 1) * T])
        ids_r.append(torch.from_numpy(ids).to(DEV))
        w_r.append(torch.from_numpy(w).to(DEV))
    outs = _emulated_layer(bank, world, X_r, ids_r, w_r, layout_T)
    assert Q.prefill_status() == 0
    store = bank["blkT"] if layout_T else bank["blk"]
    for r in range(world):
        y = outs[r].cpu().numpy()
        ref = O.prefill(list(bank["blk_np"]), bank["s2_np"], ids_np[r], w_np[r], X_r[r].float().cpu().numpy())
        assert rel_l2(y, ref) < BF16_TOL
        single = Q.moe_prefill(store, ids_r[r], w_r[r], bank["s2"], X_r[r], layout_T=layout_T)
        assert rel_l2(y, single.cpu().numpy()) < 1e-3
    # deterministic
    again = _emulated_layer(bank, world, X_r, ids_r, w_r, layout_T)
    assert all(torch.equal(a, b) for a, b in zip(outs, again))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.join(here, "..", "nemotron-super-8gb_b200"), os.path.join(here, "..")):
        sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        import ep
        import qmoe_ns as Q
        import qmoe_synth as S
        dev = torch.device("cuda", rank)
        g = S.seeded(61, dev)
        m_hat = S.unit_dir(g, dev)
        blk, s2, _ = S.expert_blocks(NE, 0.075, m_hat, g, dev)
        Q.to_T_batch(blk)
        X = S.tokens(4 * 24, m_hat, g, dev)
        el = NE // world
        layer = ep.ExpertParallelMoE(blk[rank * el:(rank + 1) * el].contiguous(), s2.float()[rank * el:(rank + 1) * el].contiguous(),
                                     n_experts=NE)
        T, k = 24, 6
        ids, w = _route(T, k, 40 + rank)
        y = layer(X[rank * T:(rank + 1) * T], torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev))
        single = Q.moe_prefill(blk, torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev), s2.float().contiguous(),
                               X[rank * T:(rank + 1) * T])
        torch.cuda.synchronize()
        q.put((rank, rel_l2(y.cpu().numpy(), single.cpu().numpy())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, repr(exc)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_layer_nccl_two_gpus():
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        assert res[r] < 1e-3
