"""The whole Nemotron-H MoE layer of a decode step on the device, without host synchronisation, and a
multi-layer step captured as one CUDA graph.

The reference's decode MoE (`moe_forward`, nem_super.py:358-392) must stop on the host once per layer
(`.tolist()` of the routed ids, :371) to drive its NVMe/RAM expert cache. With every expert resident in HBM
(expert_store.ExpertStore) nothing needs the ids on the host, so the layer is the stock
NemotronHMoE.forward (tf:722-737) over device-side parts:

    logits = x @ gate^T (fp32, tf:748-751) -> sigmoid + correction bias -> top-k ids, weights (tf:697-720)
    lat = fc1_latent_proj(x)                                     (dense_q GEMV: FP8 / NVFP4 / bf16)
    y   = routed experts(lat, ids, weights)                      (RoutedExperts: moe_decode_groups)
    out = fc2_latent_proj(y) + shared_down(relu(shared_up(x))^2) (dense_q GEMVs)

`MoELayer.forward` runs it eagerly; `DecodeGraph` records the layers of a step once as a CUDA graph over
static input/output buffers and replays it per token (one launch for the whole step). For one token on a
T-layout store, everything after the router's fp32 linear (sigmoid, bias, top-k, weights and the store
lookup of the chosen experts) is one kernel (qmoe_route_decode) instead of a dozen small torch launches.
"""
import torch
import torch.nn.functional as F

import _qmoe_lib as C
import dense_q as D
import qmoe_ns as Q
from expert_store import RoutedExperts


def linear(w, x):
    """x [..., K] -> [..., N] in x.dtype: a dense_q quantized-weight dict (FP8 / NVFP4, dense_q.py:237-247)
    runs the B200 GEMV kernels; a plain bf16 [N, K] weight with one bf16 row of x runs the bf16 GEMV
    (dq_gemv_bf16: fp32 accumulation, bf16 result, as F.linear up to the order of the fp32 sums); otherwise
    F.linear."""
    if isinstance(w, dict):
        return D.qlinear(w, x)
    if (w.dtype == torch.bfloat16 and x.dtype == torch.bfloat16 and w.dim() == 2 and w.is_contiguous()
            and x.numel() == x.shape[-1] and w.shape[1] % 8 == 0 and w.shape[1] == x.shape[-1]):
        x1 = x.reshape(1, -1).contiguous()
        y = torch.empty(1, w.shape[0], dtype=torch.bfloat16, device=x.device)
        C.call("dq_gemv_bf16", C.ptr(w), C.ptr(x1), C.dtype_code(x1), 1, w.shape[0], w.shape[1], 0, None, C.ptr(y),
               C.stream_of(x1))
        return y.view(*x.shape[:-1], w.shape[0])
    return F.linear(x, w.to(x.dtype))


def route_tokens(x, gate_w, bias, top_k=22, scaling=5.0, n_group=1, topk_group=1, norm_topk_prob=False):
    """tf:748-751 + tf:697-720 (NemotronHTopkRouter.forward, NemotronHMoE.route_tokens_to_experts) as torch
    ops on the device: x [T, hidden] -> ids int64 [T, top_k], weights f32 [T, top_k]."""
    logits = F.linear(x.reshape(-1, x.shape[-1]).to(torch.float32), gate_w.to(torch.float32))
    scores = logits.sigmoid()
    choice = scores + bias
    if n_group > 1:
        n = choice.shape[-1]
        group_scores = choice.view(-1, n_group, n // n_group).topk(2, dim=-1)[0].sum(dim=-1)
        group_idx = torch.topk(group_scores, k=topk_group, dim=-1, sorted=False)[1]
        group_mask = torch.zeros_like(group_scores)
        group_mask.scatter_(1, group_idx, 1)
        score_mask = group_mask.unsqueeze(-1).expand(-1, n_group, n // n_group).reshape(-1, n)
        choice = choice.masked_fill(~score_mask.bool(), 0.0)
    ids = torch.topk(choice, k=top_k, dim=-1, sorted=False)[1]
    w = scores.gather(1, ids)
    if norm_topk_prob:
        w = w / (w.sum(dim=-1, keepdim=True) + 1e-20)
    return ids, w * scaling


class MoELayer(torch.nn.Module):
    """One NemotronHMoE layer m (tf:663-737): gate_w [512, hidden] and bias [512] (router), fc1 [1024, hidden]
    and fc2 [hidden, 1024] (latent projections), shared_up [I, hidden] and shared_down [hidden, I] (shared
    expert, relu^2), each a dense_q dict or a plain weight; the routed experts from `store`."""

    def __init__(self, m, store, gate_w, bias, fc1, fc2, shared_up, shared_down, top_k=22, scaling=5.0,
                 n_group=1, topk_group=1, norm_topk_prob=False):
        super().__init__()
        self.gate_w = gate_w.to(torch.float32).contiguous()   # the router computes in fp32: convert once (exact)
        self.bias = bias.to(torch.float32).contiguous()
        self.fc1, self.fc2, self.shared_up, self.shared_down = fc1, fc2, shared_up, shared_down
        self.route_args = dict(top_k=top_k, scaling=scaling, n_group=n_group, topk_group=topk_group,
                               norm_topk_prob=norm_topk_prob)
        self.experts = RoutedExperts(m, store, topk=top_k)
        self._side = {}   # device index -> side stream of the one-token path
        # one-token routing in one kernel (one expert group, no renormalisation, a T-layout store)
        self.fused = n_group == 1 and not norm_topk_prob and store.layout == "T" and gate_w.shape[0] <= 1024
        if self.fused:
            dev = store.device
            self.r_ids = torch.empty(top_k, dtype=torch.int64, device=dev)
            self.r_sidx = torch.empty(top_k, dtype=torch.int32, device=dev)
            self.r_tab = torch.empty(top_k, dtype=torch.int64, device=dev)
            self.r_s2 = torch.empty(top_k, 2, dtype=torch.float32, device=dev)
            self.r_coef = torch.empty(top_k, dtype=torch.float32, device=dev)

    def route_decode(self, x):
        """One token: the router's fp32 linear, then qmoe_route_decode. Returns (ids, weights, store rows,
        block addresses, s2 rows) of the chosen experts, in order of decreasing choice."""
        st, ex = self.experts.store, self.experts
        logits = F.linear(x.to(torch.float32), self.gate_w).contiguous()
        C.call("qmoe_route_decode", C.ptr(logits), C.ptr(self.bias), self.gate_w.shape[0], self.route_args["top_k"],
               float(self.route_args["scaling"]), ex.i * st.e_local - st.lo, C.ptr(st.blocks), int(st.blocks.stride(0)),
               C.ptr(st.s2[ex.i]), C.ptr(self.r_ids), C.ptr(self.r_sidx), C.ptr(self.r_tab), C.ptr(self.r_s2),
               C.ptr(self.r_coef), C.stream_of(logits))
        return self.r_ids, self.r_coef, self.r_sidx, self.r_tab, self.r_s2

    def forward(self, hidden_states):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        if self.fused and x.shape[0] == 1 and self._fused_shared(x, x):
            return self._forward_token(x).view(shape)
        lat = linear(self.fc1, x)
        if self.fused and x.shape[0] == 1:
            _, coef, sidx, tab, s2 = self.route_decode(x)
            ex = self.experts
            y = Q.moe_decode_groups(ex.store.blocks, sidx, tab, s2, coef, lat[0], ex.h, ex.part, ex.gidx, ex.gcnt)
            y = y.view(1, -1).to(lat.dtype)
        else:
            ids, w = route_tokens(x, self.gate_w, self.bias, **self.route_args)
            y = self.experts(lat, ids, w)
        out = linear(self.fc2, y)
        if self._fused_shared(x, out):
            su, sd = self.shared_up, self.shared_down
            u2 = torch.empty(1, su["N"], dtype=torch.bfloat16, device=x.device)
            res = torch.empty_like(out)
            st = C.stream_of(x)
            C.call("dq_gemv_nvfp4_bf16", C.ptr(su["w"]), C.ptr(su["sc"]), C.ptr(su["s"]), C.ptr(x), C.dtype_code(x),
                   1, su["N"], su["K"], 1, None, C.ptr(u2), st)
            C.call("dq_gemv_nvfp4_bf16", C.ptr(sd["w"]), C.ptr(sd["sc"]), C.ptr(sd["s"]), C.ptr(u2), C.dtype_code(u2),
                   1, sd["N"], sd["K"], 2, C.ptr(out), C.ptr(res), st)
            return res.view(shape)
        u = torch.relu(linear(self.shared_up, x))
        out = out + linear(self.shared_down, u * u)
        return out.view(shape)

    def _forward_token(self, x):
        """One token with every fused part: the latent projection fc1 and the whole shared expert (up projection
        with its squared ReLU, down projection, each rounded to bf16 as the torch operators do) run on a side
        stream, forked from and joined back to the caller's stream (a CUDA graph records them as a parallel
        branch), while the router's linear, the routing kernel, the routed experts and fc2 run on the caller's
        stream; the two results are added in bf16 at the end, as the unfused layer adds them."""
        cur = torch.cuda.current_stream(x.device)
        side = self._side.get(x.device.index)
        if side is None:
            # high priority: its small GEMVs go ahead of pending CTAs of the routed layer kernel
            side = self._side[x.device.index] = torch.cuda.Stream(x.device, priority=-1)
        su, sd = self.shared_up, self.shared_down
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            lat = linear(self.fc1, x)
            lat_ready = torch.cuda.Event()
            lat_ready.record(side)
            u2 = torch.empty(1, su["N"], dtype=torch.bfloat16, device=x.device)
            C.call("dq_gemv_nvfp4_bf16", C.ptr(su["w"]), C.ptr(su["sc"]), C.ptr(su["s"]), C.ptr(x), C.dtype_code(x),
                   1, su["N"], su["K"], 1, None, C.ptr(u2), side.cuda_stream)
            shared = torch.empty(1, sd["N"], dtype=torch.bfloat16, device=x.device)
            C.call("dq_gemv_nvfp4_bf16", C.ptr(sd["w"]), C.ptr(sd["sc"]), C.ptr(sd["s"]), C.ptr(u2), C.dtype_code(u2),
                   1, sd["N"], sd["K"], 0, None, C.ptr(shared), side.cuda_stream)
        _, coef, sidx, tab, s2 = self.route_decode(x)
        cur.wait_event(lat_ready)
        ex = self.experts
        y = Q.moe_decode_groups(ex.store.blocks, sidx, tab, s2, coef, lat[0], ex.h, ex.part, ex.gidx, ex.gcnt)
        w2 = self.fc2
        if (isinstance(w2, torch.Tensor) and w2.dtype == torch.bfloat16 and lat.dtype == torch.bfloat16
                and w2.is_contiguous() and w2.shape[1] % 8 == 0):
            # fc2 on y's fp32 values rounded to bf16 as they are read (the values of y.to(bf16), without the cast)
            out = torch.empty(1, w2.shape[0], dtype=torch.bfloat16, device=x.device)
            C.call("dq_gemv_bf16", C.ptr(w2), C.ptr(y), 3, 1, w2.shape[0], w2.shape[1], 0, None, C.ptr(out),
                   cur.cuda_stream)
        else:
            out = linear(self.fc2, y.view(1, -1).to(lat.dtype))
        cur.wait_stream(side)
        if not torch.cuda.is_current_stream_capturing():   # made on the side stream, read on this one
            lat.record_stream(cur)
            u2.record_stream(cur)
            shared.record_stream(cur)
        return out + shared

    def _fused_shared(self, x, out):
        """One token, bf16 hidden states, an NVFP4 shared expert: its up projection with the squared ReLU and its
        down projection with the add are one GEMV each (dq_gemv_nvfp4_bf16; bit-identical to the torch ops)."""
        su, sd = self.shared_up, self.shared_down
        return (x.shape[0] == 1 and x.dtype == torch.bfloat16 and out.dtype == torch.bfloat16
                and isinstance(su, dict) and isinstance(sd, dict) and su["fmt"] == "nvfp4" and sd["fmt"] == "nvfp4"
                and out.is_contiguous() and x.is_contiguous())


class DecodeGraph:
    """The layers of one decode step (a token through every MoE layer in order, each layer's output feeding
    the next) recorded once as a CUDA graph: replay(x) copies x [1, hidden] into the static input, replays,
    and returns the static output buffer (valid until the next replay). Warm-up runs before capture so
    that every workspace and library handle exists before recording."""

    def __init__(self, layers, hidden, dtype=torch.bfloat16, device="cuda", warmup=2):
        self.layers = layers
        self.x = torch.zeros(1, hidden, dtype=dtype, device=device)
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._run()
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):   # the warm-up stream: its workspaces are reused
            self.out = self._run()

    def _run(self):
        h = self.x
        for layer in self.layers:
            h = layer(h)
        return h

    def replay(self, x):
        self.x.copy_(x.reshape(self.x.shape))
        self.graph.replay()
        return self.out
