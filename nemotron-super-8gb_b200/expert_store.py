"""HBM-resident routed-expert store and the experts module that runs on it.

The reference streams experts from NVMe through a RAM LRU cache into two GPU slot banks per step
(`ExpertCache`, nem_super.py:79-259) and swaps `StreamExperts` (nem_super.py:262-348) in for the
transformers `NemotronHExperts`. The whole expert file (40 MoE layers x 512 experts x 3,096,576 B =
59 GiB) fits in one B200's HBM, so here it is loaded once:

* `ExpertStore` reads the reference's own engine files (repack.py:1-7): `experts.bin`, block m*512 + e
  of layer m, expert e, laid out up_w | up_s | dn_w | dn_s (orig) or with the down half in the T layout
  when `experts.layout` says "T" (repack_T.py), and `experts_scal.npy` [40, 512, 4] f32 whose first two
  columns are weight_scale_2 of up and down. Reads run on a thread pool into pinned staging buffers and
  are copied to the device on a side stream, overlapping file reads with host-to-device copies. The store
  can be converted to the other layout in HBM at load time (qmoe_to_T / qmoe_from_T), and can hold one
  expert-parallel shard (experts lo..hi-1 of every layer) instead of all experts.
* `RoutedExperts` is the drop-in experts module: forward(hidden_states [T, 1024], top_k_index [T, k],
  top_k_weights [T, k]) -> [T, 1024] in hidden_states.dtype, as NemotronHExperts.forward / StreamExperts.forward.
  One token runs the decode kernels (moe_decode_groups on the T layout, moe_decode on the orig layout)
  with the slot indices and block addresses computed on the device - no `.tolist()` host sync as in
  nem_super.py:285 and :371. More tokens run the grouped prefill GEMM (moe_prefill).
"""
import concurrent.futures as cf
import os

import numpy as np
import torch

import _qmoe_lib as C
import qmoe_ns as Q

N_LAYERS = 40
N_EXPERTS = 512


def read_layout(directory):
    """The block layout of `experts.bin`: "T" when `experts.layout` says so, else "orig" (nem_super.py:92).
    A file being re-laid out (`experts.layout.inprogress`, repack_T.py) is refused."""
    if os.path.exists(os.path.join(directory, "experts.layout.inprogress")):
        raise C.QmoeError("experts.bin is in the middle of a layout change (experts.layout.inprogress exists)")
    p = os.path.join(directory, "experts.layout")
    if not os.path.exists(p):
        return "orig"
    lay = open(p).read().strip()
    if lay not in ("T", "orig"):
        raise C.QmoeError(f"unknown experts.layout {lay!r}")
    return lay


class ExpertStore:
    """All routed experts of the selected MoE layers resident in device memory.

    directory: holds experts.bin, experts_scal.npy and optionally experts.layout.
    layers: MoE layer indices to load (default all n_layers); layer i of the store is layers[i].
    shard: (lo, hi) expert ids of every layer to hold (expert parallelism), default all.
    layout: resident layout, "T" or "orig"; None keeps the file's. A different one is produced on the device.
    Attributes: blocks [L * E_local, BLOCK] u8 (row = layer_index * E_local + (e - lo)), s2 [L, E_local, 2]
    f32, layout, lo, hi, e_local, layers. On a CPU device nothing is converted (layout must match the file)."""

    def __init__(self, directory, device="cuda", layers=None, shard=None, layout=None, n_layers=N_LAYERS,
                 n_experts=N_EXPERTS, chunk_blocks=32, threads=4):
        self.directory = directory
        self.device = torch.device(device)
        self.n_experts = n_experts
        self.layers = list(range(n_layers)) if layers is None else [int(m) for m in layers]
        lo, hi = (0, n_experts) if shard is None else (int(shard[0]), int(shard[1]))
        if not (0 <= lo < hi <= n_experts):
            raise ValueError(f"shard {shard} outside 0..{n_experts}")
        if any(not (0 <= m < n_layers) for m in self.layers):
            raise ValueError(f"layers must lie in 0..{n_layers - 1}")
        self.lo, self.hi, self.e_local = lo, hi, hi - lo
        self.file_layout = read_layout(directory)
        self.layout = self.file_layout if layout is None else layout
        if self.layout not in ("T", "orig"):
            raise ValueError("layout must be 'T' or 'orig'")

        path = os.path.join(directory, "experts.bin")
        size = os.path.getsize(path)
        if size < n_layers * n_experts * Q.BLOCK:
            raise C.QmoeError(f"experts.bin holds {size} bytes, expected {n_layers * n_experts * Q.BLOCK} "
                              f"({n_layers} layers x {n_experts} experts x {Q.BLOCK})")
        scal = np.load(os.path.join(directory, "experts_scal.npy"))
        if scal.shape[:2] != (n_layers, n_experts) or scal.shape[2] < 2:
            raise C.QmoeError(f"experts_scal.npy has shape {scal.shape}, expected ({n_layers}, {n_experts}, 4)")
        s2 = np.ascontiguousarray(scal[self.layers][:, lo:hi, :2], dtype=np.float32)
        self.s2 = torch.from_numpy(s2).to(self.device)

        L = len(self.layers)
        self.blocks = torch.empty(L * self.e_local, Q.BLOCK, dtype=torch.uint8, device=self.device)
        self._load(path, chunk_blocks, threads)
        if self.layout != self.file_layout:
            if self.device.type != "cuda":
                raise C.QmoeError("layout conversion runs on the GPU")
            conv = Q.to_T_batch if self.layout == "T" else Q.from_T_batch
            for i in range(L):
                conv(self.layer(i))
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()

    @classmethod
    def from_tensors(cls, blocks, s2, layout, layers=None, shard=None, n_experts=N_EXPERTS):
        """A store over blocks already on the device (e.g. generated, or read by other means): blocks
        [L * E_local, BLOCK] u8 in `layout`, s2 [L, E_local, 2] f32; no file is read."""
        st = cls.__new__(cls)
        L = s2.shape[0]
        st.directory, st.device, st.n_experts = None, blocks.device, n_experts
        st.layers = list(range(L)) if layers is None else [int(m) for m in layers]
        st.lo, st.hi = (0, n_experts) if shard is None else (int(shard[0]), int(shard[1]))
        st.e_local = st.hi - st.lo
        if blocks.dtype != torch.uint8 or tuple(blocks.shape) != (L * st.e_local, Q.BLOCK) or len(st.layers) != L:
            raise ValueError("blocks must be uint8 [L * E_local, BLOCK] matching s2 [L, E_local, 2] and layers")
        if layout not in ("T", "orig"):
            raise ValueError("layout must be 'T' or 'orig'")
        st.file_layout = st.layout = layout
        st.blocks, st.s2 = blocks, s2.to(torch.float32).contiguous()
        return st

    # ------------------------------------------------------------------ loading
    def _runs(self, chunk_blocks):
        """(file block index, store row, count) runs of at most chunk_blocks contiguous blocks."""
        for i, m in enumerate(self.layers):
            first = m * self.n_experts + self.lo
            for e0 in range(0, self.e_local, chunk_blocks):
                n = min(chunk_blocks, self.e_local - e0)
                yield first + e0, i * self.e_local + e0, n

    def _load(self, path, chunk_blocks, threads):
        runs = list(self._runs(chunk_blocks))
        cuda = self.device.type == "cuda"
        nbuf = max(2, min(threads + 1, len(runs)))
        bufs = [torch.empty(chunk_blocks * Q.BLOCK, dtype=torch.uint8, pin_memory=cuda) for _ in range(nbuf)]
        done = [None] * nbuf   # CUDA event: the device copy out of staging buffer b has finished
        fd = os.open(path, os.O_RDONLY)
        copy_stream = torch.cuda.Stream(self.device) if cuda else None

        def read(b, blk, n):
            if done[b] is not None:
                done[b].synchronize()
            view = memoryview(bufs[b].numpy())[:n * Q.BLOCK]
            got, off = 0, blk * Q.BLOCK
            while got < n * Q.BLOCK:
                k = os.preadv(fd, [view[got:]], off + got)
                if k <= 0:
                    raise C.QmoeError(f"short read of experts.bin at block {blk}")
                got += k
            return b

        try:
            with cf.ThreadPoolExecutor(max(1, threads)) as pool:
                pending = {}
                for r, (blk, row, n) in enumerate(runs):
                    if r < nbuf:
                        pending[r] = pool.submit(read, r % nbuf, blk, n)
                for r, (blk, row, n) in enumerate(runs):
                    b = pending.pop(r).result()
                    dst = self.blocks[row:row + n].view(-1)
                    if cuda:
                        with torch.cuda.stream(copy_stream):
                            dst.copy_(bufs[b][:n * Q.BLOCK], non_blocking=True)
                            ev = torch.cuda.Event()
                            ev.record(copy_stream)
                        done[b] = ev
                    else:
                        dst.copy_(bufs[b][:n * Q.BLOCK])
                    nxt = r + nbuf
                    if nxt < len(runs):
                        blk2, _, n2 = runs[nxt]
                        pending[nxt] = pool.submit(read, b, blk2, n2)
        finally:
            os.close(fd)
        if cuda:
            torch.cuda.current_stream(self.device).wait_stream(copy_stream)

    # ------------------------------------------------------------------ addressing
    def layer(self, i):
        """Store rows of loaded layer i: [E_local, BLOCK] u8 (a view)."""
        return self.blocks[i * self.e_local:(i + 1) * self.e_local]

    def index(self, m):
        """Store layer index of MoE layer m."""
        try:
            return self.layers.index(m)
        except ValueError:
            raise KeyError(f"MoE layer {m} is not loaded") from None

    def slot_index(self, i, ids):
        """int32 store rows of experts `ids` (global ids, on the device) of loaded layer i."""
        return (ids.to(torch.int64) - self.lo + i * self.e_local).to(torch.int32)

    def block_addresses(self, sidx):
        """int64 device addresses of the blocks at store rows sidx."""
        return sidx.to(torch.int64) * self.blocks.stride(0) + self.blocks.data_ptr()


class RoutedExperts(torch.nn.Module):
    """Replacement of NemotronHExperts for MoE layer m (nem_super.py:262-348, StreamExperts), computing on an
    ExpertStore that holds all experts of the layer: forward(hidden_states [T, 1024], top_k_index [T, k]
    int, top_k_weights [T, k]) -> [T, 1024] in hidden_states.dtype = sum over k of weights * expert(x).
    T = 1 runs the decode kernels; T > 1 the grouped prefill GEMM."""

    def __init__(self, m, store, topk=22):
        super().__init__()
        if store.e_local != store.n_experts:
            raise ValueError("RoutedExperts needs every expert of the layer; use ep.ExpertParallelMoE for a shard")
        self.m, self.store, self.topk = m, store, topk
        self.i = store.index(m)
        dev = store.device
        self.h = torch.empty(topk, Q.INTER, device=dev)
        self.o = torch.empty(topk, Q.LAT, device=dev)
        self.part = torch.empty(Q.GROUP_CFG["KS"], topk, Q.LAT, device=dev)
        self.gidx = torch.empty(topk, Q.G_DN, dtype=torch.int32, device=dev)
        self.gcnt = torch.empty(topk, dtype=torch.int32, device=dev)

    def forward(self, hidden_states, top_k_index, top_k_weights):
        st = self.store
        T, k = top_k_index.shape
        if k > self.topk:
            raise ValueError(f"top-k {k} exceeds the module's {self.topk}")
        if T == 1:
            ids = top_k_index[0]
            sidx = st.slot_index(self.i, ids).contiguous()
            s2 = st.s2[self.i].index_select(0, ids.to(torch.int64)).contiguous()
            coef = top_k_weights[0].to(torch.float32).contiguous()
            x = hidden_states[0]
            if st.layout == "T":
                y = Q.moe_decode_groups(st.blocks, sidx, st.block_addresses(sidx), s2, coef, x, self.h, self.part,
                                        self.gidx, self.gcnt)
            else:
                y = Q.moe_decode(st.blocks, sidx, s2, coef, x, self.h, self.o)
            return y.view(1, -1).to(hidden_states.dtype)
        y = Q.moe_prefill(st.layer(self.i), top_k_index, top_k_weights, st.s2[self.i], hidden_states,
                          layout_T=st.layout == "T")
        return y.to(hidden_states.dtype)


def write_engine_files(directory, blocks, scal, layout="orig"):
    """Write `experts.bin` (blocks [n_layers * n_experts, BLOCK] u8, block m*n_experts + e), `experts_scal.npy`
    (scal [n_layers, n_experts, 4] f32) and `experts.layout` in the reference's engine-file format
    (repack.py:1-7). For tests and for converting synthetic stores; the real files come from repack.py."""
    os.makedirs(directory, exist_ok=True)
    arr = blocks.cpu().numpy() if isinstance(blocks, torch.Tensor) else np.asarray(blocks)
    arr.astype(np.uint8, copy=False).tofile(os.path.join(directory, "experts.bin"))
    np.save(os.path.join(directory, "experts_scal.npy"), np.asarray(scal, dtype=np.float32))
    with open(os.path.join(directory, "experts.layout"), "w") as f:
        f.write(layout + "\n")
