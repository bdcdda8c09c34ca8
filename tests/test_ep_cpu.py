"""Expert-parallel exchange protocol (nemotron-super-8gb_b200/ep.py) on CPU ranks over gloo, world size 2.

The device steps (pack, local experts, combine) are replaced by the oracle's restatements (oracle.ep_pack,
oracle.prefill, oracle.ep_combine) so that the host logic — block shapes, the three all_to_all exchanges,
the id/weight packing, the rank-order combine — runs without a GPU. Each rank's result must equal the
single-process oracle layer over all experts for that rank's tokens."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import vectors as V

NE, K, T = 8, 3, 5


class OracleOps:
    """CPU stand-ins for ep.CudaOps, built on the oracle (test infrastructure)."""

    def __init__(self, blocks_local):
        self.blocks = blocks_local

    def pack(self, x, ids, weights, n_experts, world):
        from oracle import oracle as O
        sx, si, sw, row_of, cnt = O.ep_pack(x.numpy(), ids.numpy(), weights.numpy(), n_experts, world)
        meta = np.concatenate([si, sw.view(np.int32)], axis=2)
        return torch.from_numpy(sx), torch.from_numpy(meta), torch.from_numpy(row_of), torch.from_numpy(cnt)

    def local(self, store, s2, recv_x, recv_meta, layout_T):
        from oracle import oracle as O
        k = recv_meta.shape[1] // 2
        ids = recv_meta[:, :k].numpy()
        w = recv_meta[:, k:].contiguous().view(torch.float32).numpy()
        out = O.prefill(self.blocks, s2.numpy(), ids, w, recv_x.numpy())
        return torch.from_numpy(out.astype(np.float32))

    def combine(self, recv_part, row_of):
        from oracle import oracle as O
        return torch.from_numpy(O.ep_combine(recv_part.numpy().astype(np.float64), row_of.numpy()))


def _inputs(rank):
    rng = np.random.default_rng(1000 + rank)
    X = V.bf16_round(rng.normal(0, 0.5, (T, 1024)).astype(np.float32))
    ids = np.stack([rng.permutation(NE)[:K] for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, (T, K)).astype(np.float32)
    return X, ids, w


def _bank():
    rng = np.random.default_rng(77)
    blocks = [V.rand_block(500 + e) for e in range(NE)]
    s2 = rng.uniform(0.002, 0.02, (NE, 2)).astype(np.float32)
    return blocks, s2


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "nemotron-super-8gb_b200"))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import ep
        blocks, s2 = _bank()
        lo, hi = ep.shard_bounds(NE, world, rank)
        store = torch.zeros(hi - lo, 8, dtype=torch.uint8)   # shape check only; OracleOps reads the blocks
        layer = ep.ExpertParallelMoE(store, torch.from_numpy(s2[lo:hi]), n_experts=NE, ops=OracleOps(blocks[lo:hi]))
        X, ids, w = _inputs(rank)
        y = layer(torch.from_numpy(X), torch.from_numpy(ids), torch.from_numpy(w))
        q.put((rank, y.numpy()))
        dist.destroy_process_group()
    except Exception as exc:   # reported to the parent
        q.put((rank, repr(exc)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_ep_protocol_world2_matches_single_process():
    from oracle import oracle as O
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, y = q.get(timeout=300)
        got[r] = y
    for p in procs:
        p.join(timeout=60)
    blocks, s2 = _bank()
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
        X, ids, w = _inputs(r)
        ref = O.prefill(blocks, s2, ids, w, X)
        assert np.linalg.norm(got[r] - ref) / np.linalg.norm(ref) < 1e-6


def test_ep_pack_oracle_contract():
    """Pack/combine restatement: every (token, destination) with a local expert appears once, in token order,
    and combining per-rank partials of 1 reproduces the number of ranks each token reached."""
    from oracle import oracle as O
    X, ids, w = _inputs(0)
    sx, si, sw, row_of, cnt = O.ep_pack(X, ids, w, NE, 4)
    el = NE // 4
    for d in range(4):
        rows = [t for t in range(T) if ((ids[t] // el) == d).any()]
        assert cnt[d] == len(rows)
        assert [int(r) for r in row_of[d] if r >= 0] == list(range(len(rows)))
        for r, t in enumerate(rows):
            assert np.array_equal(sx[d, r], X[t])
            assert np.array_equal(si[d, r], np.where(ids[t] // el == d, ids[t] - d * el, -1))
        assert (si[d, cnt[d]:] == -1).all()
    part = np.ones((4, T, 2))
    hits = O.ep_combine(part, row_of)[:, 0]
    assert np.array_equal(hits, np.array([len(set(ids[t] // el)) for t in range(T)], dtype=np.float64))


def test_ep_module_rejects_wrong_shard():
    """A rank's store must hold exactly n_experts / world experts."""
    import ep
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        with pytest.raises(ValueError):
            ep.ExpertParallelMoE(torch.zeros(3, 8, dtype=torch.uint8), torch.zeros(3, 2), n_experts=8)
        layer = ep.ExpertParallelMoE(torch.zeros(8, 8, dtype=torch.uint8), torch.zeros(8, 2), n_experts=8)
        assert (layer.world, layer.rank, layer.e_local) == (1, 0, 8)
    finally:
        dist.destroy_process_group()
