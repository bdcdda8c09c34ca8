"""Expert-parallel routed-expert layer over torch.distributed (NCCL between GPUs of one node).

The reference runs all 512 experts of a layer on one GPU (nem_super.py:278-348, StreamExperts.forward).
Here expert e of a layer lives on rank e // (n_experts // world). One forward of T tokens per rank:

  1. pack (libqmoe_b200 qmoe_ep_dispatch_pack): per destination rank d, the tokens with >= 1 expert on d,
     in token order, as fixed-size blocks of T rows (activations; block-local ids, -1 for experts elsewhere;
     routing weights);
  2. dispatch: all_to_all of the activation blocks and of the id/weight blocks;
  3. local experts: qmoe_prefill_grouped over the world*T received rows (id -1 skipped), which sums each
     row's local experts in k order;
  4. combine: all_to_all of the partial outputs back to their source ranks, then qmoe_ep_combine sums each
     token's partials in rank order.

Fixed T-row blocks keep the split sizes on the device (no host synchronisation); with 22 of 512 experts per
token a token reaches nearly every rank, so the bound is nearly tight. The data-moving steps are injectable
(`ops`) so that the exchange protocol runs on CPU ranks (gloo) with reference implementations in tests.
"""
import torch
import torch.distributed as dist

import _qmoe_lib as C
import qmoe_ns as Q

LAT = Q.LAT


class CudaOps:
    """The device steps of an expert-parallel forward, on libqmoe_b200."""

    def pack(self, x, ids, weights, n_experts, world):
        T, k = ids.shape
        dev = x.device
        x = x.contiguous()
        ids32 = ids.to(torch.int32).contiguous()
        w32 = weights.to(torch.float32).contiguous()
        send_x = torch.empty((world, T, LAT), dtype=x.dtype, device=dev)
        send_meta = torch.empty((world, T, 2 * k), dtype=torch.int32, device=dev)
        row_of = torch.empty((world, T), dtype=torch.int32, device=dev)
        send_cnt = torch.empty(world, dtype=torch.int32, device=dev)
        C.call("qmoe_ep_dispatch_pack", C.ptr(x), C.dtype_code(x), C.ptr(ids32), C.ptr(w32), T, k, n_experts, world,
               C.ptr(send_x), C.ptr(send_meta), C.ptr(row_of), C.ptr(send_cnt), C.stream_of(x))
        return send_x, send_meta, row_of, send_cnt

    def local(self, store, s2, recv_x, recv_meta, layout_T):
        rows, k2 = recv_meta.shape
        k = k2 // 2
        ids = recv_meta[:, :k].contiguous()
        w = recv_meta[:, k:].contiguous().view(torch.float32)
        return Q.moe_prefill(store, ids, w, s2, recv_x, layout_T=layout_T)

    def combine(self, recv_part, row_of):
        world, T, _ = recv_part.shape
        out = torch.empty((T, LAT), dtype=torch.float32, device=recv_part.device)
        C.call("qmoe_ep_combine", C.ptr(recv_part.contiguous()), C.ptr(row_of), T, world, C.ptr(out),
               C.stream_of(recv_part))
        return out


class ExpertParallelMoE:
    """One MoE layer's routed experts sharded over the ranks of `group`.

    store_local [n_experts // world, >= BLOCK] u8 holds this rank's experts (rank r: experts
    r*E_local .. (r+1)*E_local - 1), s2_local [E_local, 2] their weight_scale_2 pairs."""

    def __init__(self, store_local, s2_local, n_experts=512, group=None, layout_T=True, ops=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        self.e_local = n_experts // self.world
        if store_local.shape[0] != self.e_local:
            raise ValueError(f"store_local holds {store_local.shape[0]} experts, expected {self.e_local}")
        self.n_experts = n_experts
        self.store = store_local
        self.s2 = s2_local
        self.layout_T = layout_T
        self.ops = ops if ops is not None else CudaOps()

    def forward(self, x, top_k_index, top_k_weights, marks=None):
        """x [T, 1024], top_k_index [T, k] global expert ids, top_k_weights [T, k] -> fp32 [T, 1024]:
        sum over k of weight * expert(x), the local experts' terms summed in k order on their rank and the
        ranks' partials summed in rank order. Every rank must call with the same T and k.
        marks: a list that receives (phase, CUDA event) after each phase ("start", "pack", "dispatch",
        "experts", "return", "combine"), recorded on the current stream, for timing the exchange."""
        T, k = top_k_index.shape
        world = self.world

        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))

        mark("start")
        send_x, send_meta, row_of, _ = self.ops.pack(x, top_k_index, top_k_weights, self.n_experts, world)
        mark("pack")
        recv_x = torch.empty_like(send_x)
        recv_meta = torch.empty_like(send_meta)
        dist.all_to_all_single(recv_x, send_x, group=self.group)
        dist.all_to_all_single(recv_meta, send_meta, group=self.group)
        mark("dispatch")
        part = self.ops.local(self.store, self.s2, recv_x.view(world * T, LAT), recv_meta.view(world * T, 2 * k),
                              self.layout_T)
        part = part.view(world, T, LAT)
        mark("experts")
        recv_part = torch.empty_like(part)
        dist.all_to_all_single(recv_part, part, group=self.group)
        mark("return")
        out = self.ops.combine(recv_part, row_of)
        mark("combine")
        return out

    __call__ = forward


def shard_bounds(n_experts, world, rank):
    """Experts [lo, hi) that rank `rank` holds."""
    e_local = n_experts // world
    return rank * e_local, (rank + 1) * e_local
