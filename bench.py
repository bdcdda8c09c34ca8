"""Benchmark of the B200 routed-expert path (BASELINE metric: MoE decode us/token and HBM GB/s; prefill tok/s
at 1/2/4/8 B200).

Default workload: full 40-layer routed-expert decode, bs = 1, one B200. All
40 x 512 synthetic NVFP4 experts (59 GiB, T layout) are resident in HBM; per-layer live fractions are
spread uniformly over 1-16.5%. A step is one token: 40 layer calls of the decode-step routed-expert
forward (up GEMV + ReLU^2, live-group compaction, live-group down GEMV, fixed-order combine; fp32
accumulation as the reference), each on its own routed top-22 experts. The per-token inputs rotate over a
64-token stream, and one token reads ~1.5 GB of distinct expert bytes, far more than the 126 MB L2, so no
step is served from L2.

  value : device time of K steps replayed from CUDA graphs (inputs resident in HBM), us/token.
  e2e   : the same step through the public API with host buffers, layer by layer as the model runs it: per
          layer, the H2D copy of that layer's routed inputs from pinned host memory, the layer call, and the
          D2H copy of its output (layer m+1's input depends on layer m's output in the real model).
  roofline: the fused layer kernel (decode_layer_kernel + its finish kernel), per layer, from the CUDA events
          of the timed region, against the measured HBM copy bandwidth (MEASURED_PEAKS.json).
  prefill (N = 1): BASELINE config 3, one 512-expert layer, T = 2048 (and T = 64) tokens through
          qmoe_prefill_grouped: tokens/s, roofline, e2e, CPU baseline, clocks.
  ep (every N): BASELINE config 4, expert parallelism over the N ranks (512 / N experts of every layer per
          rank), 40 layers, batched decode of 64 tokens per rank and prefill of 8192 tokens per rank: tokens/s
          over all ranks (max-over-ranks device time) and the measured share of the all-to-all exchanges.

--impl reference: the reference's fp32 CPU expert path (nem_super.py:342-346), as restated by the oracle
port, on the host cores: each step one token of config 1's own store and token stream, all 40 layers x 22
experts, the tokens the repo arm times.
--gpus N (torchrun): bs = 1 decode does not shard: N independent replicas (value = total tokens of all
ranks / max-over-ranks time); the ep sub-record is the sharded path.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nemotron-super-8gb_b200"))
sys.path.insert(0, ROOT)

METRIC = "MoE decode us/token (40-layer routed-expert decode, bs=1)"
# One decode_layer_kernel launch at K = 22 from a single-launch ncu capture (`--layers 2` store, 13th launch):
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) and the bytes its loads moved from L2 to the SMs
# (l1tex__m_xbar2l1tex_read_bytes.sum). That layer's live fraction is below the mean, so the line reports the
# DRAM/requested ratio applied to the mean layer's algorithmic bytes. ncu cannot run inside the timed bench,
# so the figures are carried here.
LAYER_TRAFFIC_NCU = {"dram_bytes": 34996480, "requested_bytes": 35736640}
N_LAYERS, NE, K = 40, 512, 22
N_TOK = 64


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "dense", "prefill", "ep", "decode_step"])
    ap.add_argument("--ep-t", type=int, default=64, help="ep workload: tokens per rank per step (config 4 decode batch)")
    ap.add_argument("--prefill-t", type=int, default=2048, help="prefill workload: tokens per call (config 3)")
    ap.add_argument("--prefill-layout", default="orig", choices=["orig", "T"],
                    help="prefill workload: store layout (T: the down halves are converted inside the call)")
    ap.add_argument("--no-prefill", action="store_true", help="decode workload: skip the prefill sub-record")
    ap.add_argument("--no-ep", action="store_true", help="decode workload: skip the expert-parallel sub-record")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """SM clock and throttle reasons sampled during the timed region: nvidia-smi (the recipe's query, every
    100 ms) and, so that regions of a few milliseconds still get samples, NVML read every 5 ms by a thread.
    Both only read the GPU's state."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.nv = []          # (sm MHz, max MHz, reason names)
        self.p = None
        self.nv_t = None
        self.stop_ev = threading.Event()
        self.nv0 = 0

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.p = None
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
            first = threading.Event()

            def poll():
                while not self.stop_ev.is_set():
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                        r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.nv.append((float(sm), float(mx), [n for n, b in bits.items() if r & b]))
                    except Exception:
                        break
                    finally:
                        first.set()
                    time.sleep(0.005)

            self.nv_t = threading.Thread(target=poll, daemon=True)
            self.nv_t.start()
            first.wait(timeout=2.0)
        except Exception:
            self.nv_t = None
        t0 = time.time()   # let nvidia-smi print its first row, so that it samples the whole region
        while self.p is not None and not self.rows and time.time() - t0 < 1.5 and self.p.poll() is None:
            time.sleep(0.01)
        self.nv0 = max(len(self.nv) - 1, 0)   # NVML samples from the last one before the region on

    def _read(self):
        for line in self.p.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        n_smi = len(self.rows)
        self.stop_ev.set()
        if self.nv_t is not None:
            self.nv_t.join(timeout=2)
            try:
                import pynvml
                pynvml.nvmlShutdown()
            except Exception:
                pass
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()
            self.t.join(timeout=2)
        rows = self.rows[:n_smi]
        sm = [float(r[1]) for r in rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for i, n in enumerate(self.NAMES):
                if len(r) > 5 + i and r[5 + i] == "Active":
                    reasons.add(n)
        for s, m, rs in self.nv[self.nv0:]:
            sm.append(s)
            mx.append(m)
            reasons.update(rs)
        if self.p is None and self.nv_t is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "nvidia_smi_samples": len(rows),
                "nvml_samples": len(self.nv) - self.nv0}


def build_store(torch, S, dev, n_layers, seed, layout_T=True):
    """HBM-resident expert store: [n_layers*512, BLOCK] u8 in the T layout (converted with qmoe_to_T) or,
    with layout_T=False, the orig layout; s2 [n_layers, 512, 2], per-layer m_hat and router, generated in
    batches on the device."""
    import qmoe_ns as Q
    g = S.seeded(seed, dev)
    store = torch.empty(n_layers * NE, S.BLOCK, dtype=torch.uint8, device=dev)
    s2 = torch.empty(n_layers, NE, 2, dtype=torch.float32, device=dev)
    p_l = S.layer_live_fractions(n_layers) if n_layers > 1 else [0.075]
    m_hats, routers = [], []
    B = 32
    for m in range(n_layers):
        m_hat = S.unit_dir(g, dev)
        m_hats.append(m_hat)
        routers.append(S.router(g, dev))
        for e0 in range(0, NE, B):
            blk, s2b, _ = S.expert_blocks(B, p_l[m], m_hat, g, dev)
            store[m * NE + e0:m * NE + e0 + B].copy_(blk)
            s2[m, e0:e0 + B] = s2b
            del blk
        if layout_T:
            Q.to_T_batch(store[m * NE:(m + 1) * NE])
    torch.cuda.synchronize()
    return store, s2, m_hats, routers, p_l


def make_tokens(torch, S, dev, store, s2, m_hats, routers, n_tok, seed):
    """Per token and layer: x bf16 [1024], routed ids, weights -> packed per-token inputs."""
    g = S.seeded(seed + 1, dev)
    L = len(m_hats)
    X = torch.empty(n_tok, L, S.LAT, dtype=torch.bfloat16, device=dev)
    IDS = torch.empty(n_tok, L, K, dtype=torch.int64, device=dev)
    W = torch.empty(n_tok, L, K, dtype=torch.float32, device=dev)
    for m in range(L):
        x = S.tokens(n_tok, m_hats[m], g, dev)
        ids, w = S.route(x, *routers[m])
        X[:, m] = x
        IDS[:, m] = ids
        W[:, m] = w
    base = store.data_ptr()
    layer = torch.arange(L, device=dev).view(1, L, 1)
    SIDX = (layer * NE + IDS).to(torch.int32)
    TAB = base + SIDX.to(torch.int64) * S.BLOCK
    S2 = s2[layer.expand(n_tok, L, K), IDS]
    return dict(X=X.contiguous(), SIDX=SIDX.contiguous(), TAB=TAB.contiguous(), S2=S2.contiguous(),
                W=W.contiguous(), IDS=IDS)


class DecodeStep:
    """One token of 40-layer decode over static device buffers, capturable in a CUDA graph."""

    def __init__(self, torch, dev, store, L):
        import _qmoe_lib as C
        import qmoe_ns as Q
        self.C, self.Q, self.torch, self.L = C, Q, torch, L
        self.store = store
        self.h = torch.empty(L, K, Q.INTER, device=dev)
        self.part = torch.empty(L, K, Q.LAT, device=dev)
        self.gidx = torch.empty(L, K, 168, dtype=torch.int32, device=dev)
        self.gcnt = torch.empty(L, K, dtype=torch.int32, device=dev)
        self.Y = torch.empty(L, Q.LAT, device=dev)
        nbytes = int(C.lib().qmoe_decode_groups_workspace_bytes(K))
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self.fn = C.lib().qmoe_decode_groups

    def launch(self, X, SIDX, TAB, S2, W, stream):
        C, Q = self.C, self.Q
        sp, sb, ns = self.store.data_ptr(), int(self.store.stride(0)), int(self.store.shape[0])
        for m in range(self.L):
            rc = self.fn(sp, sb, ns, SIDX[m].data_ptr(), TAB[m].data_ptr(), S2[m].data_ptr(), W[m].data_ptr(),
                         X[m].data_ptr(), 1, K, self.h[m].data_ptr(), self.gidx[m].data_ptr(), self.gcnt[m].data_ptr(),
                         self.part[m].data_ptr(), self.Y[m].data_ptr(), self.ws.data_ptr(), self.ws.numel(), stream)
            if rc != 0:
                raise C.QmoeError(f"qmoe_decode_groups: {C.status_string(rc)}")


def algorithmic_bytes(torch, step_bufs, L):
    """Per-token algorithmic HBM bytes: per layer sum_j [UPB + 1024*live groups_j + 512*live neurons_j]
    + x (2 KB) + y (4 KB); h stays on chip in an ideal fused kernel."""
    live = step_bufs.h > 0
    lm = live.view(L, K, 168, 16)
    groups = int(lm.any(-1).sum())
    neurons = int(live.sum())
    return L * K * 1548288 + 1024 * groups + 512 * neurons + L * (2048 + 4096), groups, neurons


def host_cores():
    """Cores this process may run on (torchrun sets OMP_NUM_THREADS=1 per rank; the CPU baseline runs on rank 0
    alone and should use all of them)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def decode_token_inputs(store, s2_host, T, tok, L, layout_T):
    """Host copies of token `tok`'s routed experts, layer by layer: [(22 orig-layout blocks, s2 [22,2], coef [22],
    x [1024] f32)]. T-layout blocks are converted back with the oracle's from_T (the reference's prompt path
    converts them with from_T_fast before its fp32 CPU path, nem_super.py:324-328)."""
    import numpy as np
    from oracle import oracle as O
    out = []
    for m in range(L):
        ids = T["IDS"][tok, m]
        rows = store.index_select(0, m * NE + ids).cpu().numpy()
        blocks = [O.from_T(b) for b in rows] if layout_T else list(rows)
        out.append((blocks, np.ascontiguousarray(s2_host[m][ids.cpu().numpy()]), T["W"][tok, m].cpu().numpy(),
                    T["X"][tok, m].float().cpu().numpy()))
    return out


def decode_cpu_token(layers, threads):
    """The reference's fp32 CPU expert path (nem_super.py:342-346: block_deq, relu(U x)^2, D h, x coef, summed) as
    restated by the oracle, over one token's layers on `threads` host threads. Returns the compute seconds (the
    host copies of the blocks are made before, untimed)."""
    from oracle import oracle as O
    t = 0.0
    for blocks, s2, coef, x in layers:
        t0 = time.perf_counter()
        O.cpu_layer_fp32(blocks, s2, coef, x, layoutT=False, nthreads=threads)
        t += time.perf_counter() - t0
    return t


def decode_config(L, world):
    """The `config` of the decode line, the same for the repo arm and the reference arm."""
    return {"workload": "config1: 40-layer routed-expert decode, bs=1, HBM-resident T-layout store", "layers": L,
            "experts": NE, "top_k": K, "tokens_rotated": N_TOK, "l2": "inputs larger than L2 (1.5 GB/token)",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}


def cpu_baseline(store, s2_host, T, L, tok, threads=0):
    """The reference arm's code on one token of the timed stream (token `tok`, all layers x 22 experts)."""
    n = host_cores() if threads <= 0 else threads
    layers = decode_token_inputs(store, s2_host, T, tok, L, layout_T=True)
    dt = decode_cpu_token(layers, n)
    return {"value": round(dt * 1e6, 1), "unit": "us/token", "cores": n, "kind": "port",
            "sample": f"token {tok} of the 64-token stream, all {L} layers x {K} routed experts "
                      f"(the reference arm's code and inputs), {dt / L * 1e3:.1f} ms/layer"}


def run_reference(args):
    """--impl reference: the oracle port of the reference's fp32 CPU path, rank 0 only."""
    import numpy as np
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload == "prefill":
        return run_reference_prefill(args)
    if args.workload == "dense":
        return run_reference_dense(args)
    if args.workload == "ep":
        print(json.dumps({"impl": "reference", "unavailable": "the reference engine has no expert parallelism: it "
                          "runs every expert on one GPU (see --workload prefill / decode for its paths)"}), flush=True)
        return
    import torch
    import qmoe_synth as S
    n = host_cores()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    # config 1's own store and token stream, generated on the device exactly as the repo arm generates them
    # (same seeds, same draws; the orig layout, which the reference's CPU path reads), then copied to the host
    # token by token. The timed steps are the tokens the repo arm's timed steps replay.
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    L = args.layers
    store, s2, m_hats, routers, _ = build_store(torch, S, dev, L, seed=1000, layout_T=False)
    T = make_tokens(torch, S, dev, store, s2, m_hats, routers, N_TOK, seed=2000)
    s2_host = s2.cpu().numpy()
    samples = []
    t_all = time.perf_counter()
    for it in range(args.warmup + args.steps):
        layers = decode_token_inputs(store, s2_host, T, it % N_TOK, L, layout_T=False)
        dt = decode_cpu_token(layers, n)
        if it >= args.warmup:
            samples.append(dt * 1e6)
        if time.perf_counter() - t_all > 240:   # a bound on the whole run; the line reports the steps timed
            break
    if not samples:
        print(json.dumps({"impl": "reference", "unavailable": "the warm-up steps used up the 240 s bound of the "
                          "CPU path; run with fewer warm-up steps"}), flush=True)
        return
    v = float(np.mean(samples))
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 1), "unit": "us/token", "n_gpus": args.gpus,
            "steps": len(samples), "warmup": args.warmup, "ms_per_step": round(v / 1e3, 3), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": decode_config(L, world),
            "cpu_baseline": {"value": round(v, 1), "unit": "us/token", "cores": n, "kind": "port",
                             "sample": f"per step one token of the 64-token stream (tokens {args.warmup} onwards, as "
                                       f"the repo arm times), all {L} layers x {K} routed experts"},
            "e2e": {"value": round(v, 1), "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_prefill(args):
    """--impl reference --workload prefill: the reference's prompt path (prefill_cpu_reference) on the host
    cores for the same workload as the prefill arm: T tokens drawn as in config 0, routed top-22 of 512 by the
    synthetic router, one layer; each step times a bounded sample of the experts hit, scaled to all."""
    import numpy as np
    import torch
    import qmoe_synth as S
    T = args.prefill_t
    g = S.seeded(303, "cpu")
    m_hat = S.unit_dir(g, "cpu")
    router = S.router(g, "cpu")
    X = S.tokens(T, m_hat, S.seeded(404, "cpu"), "cpu")
    ids, w = S.route(X, *router)
    ids = ids.to(torch.int32).numpy()
    w = w.float().numpy()
    Xf = X.float().numpy()
    uniq = int(np.unique(ids).size)
    cache = {}
    s2 = np.zeros((NE, 2), np.float32)

    def block_of(e):   # synthetic expert blocks, generated once per expert sampled
        if e not in cache:
            blk, s2b, _ = S.expert_blocks(1, 0.0875, m_hat, S.seeded(5000 + e, "cpu"), "cpu")
            cache[e] = blk[0].numpy()
            s2[e] = s2b[0].numpy()
        return cache[e]
    samples = []
    n = host_cores()
    sample = ""
    for it in range(args.warmup + args.steps):
        v, n, sample = prefill_cpu_reference(block_of, s2, ids, w, Xf, budget_s=10.0, threads=n, max_experts=24)
        if it >= args.warmup:
            samples.append(v)
    v = float(np.mean(samples))
    line = {"impl": "reference", "metric": PREFILL_METRIC, "value": round(v, 1), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": len(samples), "warmup": args.warmup, "ms_per_step": round(T / v * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config3: prefill T={T}", "T": T, "top_k": K, "experts": NE,
                       "unique_experts": uniq, "layout": "orig"},
            "cpu_baseline": {"value": round(v, 1), "unit": "tokens/s", "cores": n, "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


DENSE_METRIC = "dense_q GEMV us per call (config 2 sweep, bs=1)"


def run_reference_dense(args):
    """--impl reference --workload dense: the dense GEMVs' CPU restatement (dense_cpu_reference: dequantize
    and multiply, one thread) over the config 2 shapes at bs = 1, one weight copy per shape drawn on the host
    as the dense arm draws them (N(0, 0.02) before quantization, bf16 x ~ N(0, 1))."""
    import numpy as np
    import torch
    import qmoe_synth as S
    g = S.seeded(77, "cpu")
    weights = []
    for fmt, N, K in DENSE_SHAPES:
        wf = torch.randn(N, K, generator=g) * 0.02
        if fmt == "fp8":
            codes, s_ = S.quantize_fp8(wf)
            q = {"fmt": "fp8", "w": codes.numpy(), "s": s_.reshape(1).numpy(), "N": N, "K": K}
        else:
            codes, sc, s2 = S.quantize_nvfp4(wf)
            q = {"fmt": "nvfp4", "w": codes.numpy(), "sc": sc.numpy(), "s": s2.reshape(1).numpy(), "N": N, "K": K}
        del wf
        weights.append((q, torch.randn(K, generator=g).to(torch.bfloat16).float().numpy()))
    samples = []
    for it in range(args.warmup + args.steps):
        us = dense_cpu_reference(weights, budget_s=120.0)
        if it >= args.warmup and all(u is not None for u in us):
            samples.append(sum(us))
    if not samples:
        print(json.dumps({"impl": "reference", "unavailable": "the dense CPU restatement did not finish one sweep of "
                          "the shapes within its time budget"}), flush=True)
        return
    v = float(np.mean(samples))
    line = {"impl": "reference", "metric": DENSE_METRIC, "value": round(v, 1), "unit": "us (sum of shapes)",
            "n_gpus": args.gpus, "steps": len(samples), "warmup": args.warmup, "ms_per_step": round(v / 1e3, 3),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f64 (oracle)",
            "data": "synthetic",
            "config": {"workload": "config2: dense_q GEMV sweep", "shapes": [list(s_) for s_ in DENSE_SHAPES]},
            "cpu_baseline": {"value": round(v, 1), "unit": "us (sum of shapes)", "cores": 1, "kind": "port",
                             "sample": "each bs=1 shape once per step: oracle dequantize + matrix-vector product"},
            "e2e": {"value": round(v, 1), "unit": "us (sum of shapes)", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


DENSE_SHAPES = [("fp8", 4096, 4096), ("fp8", 12288, 4096), ("fp8", 4096, 8192), ("fp8", 131072, 4096),
                ("nvfp4", 2688, 4096), ("nvfp4", 4096, 2688)]


def dense_cpu_reference(weights, budget_s=20.0):
    """The dense GEMVs on the host: the oracle's C restatement of dense_q.py:179-188 (dequantize, then the
    matrix-vector product; one thread, fp64 accumulation) for each (q, x) of `weights`, q the quantized-weight
    dict with numpy arrays. Returns the per-call times in microseconds (a shape whose turn comes after the
    time budget is spent is skipped: None)."""
    import numpy as np
    from oracle import oracle as O
    out = []
    t_all = time.perf_counter()
    for q, x in weights:
        if time.perf_counter() - t_all > budget_s:
            out.append(None)
            continue
        t0 = time.perf_counter()
        O.dense(q["fmt"], q["w"], q.get("sc"), float(np.asarray(q["s"]).reshape(-1)[0]), q["N"], q["K"], x)
        out.append((time.perf_counter() - t0) * 1e6)
    return out


def run_dense(args):
    """dense_q GEMVs at bs = 1 (and M = 2), FP8 per-tensor and NVFP4 weights drawn
    N(0, 0.02) before quantization, bf16 x ~ N(0, 1). Each shape rotates over enough weight copies that the
    bytes of one rotation exceed L2; time per call from CUDA events over graph replays."""
    import torch
    import dense_q as D
    import qmoe_synth as S
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    hbm, peak_kind = peaks()
    g = S.seeded(77, dev)
    st = torch.cuda.Stream()
    res = []
    cpu_q = []          # one weight copy per shape on the host, for the CPU baseline
    launches = 0
    for fmt, N, K in DENSE_SHAPES:
        wbytes = N * K if fmt == "fp8" else N * K // 2 + N * K // 16
        copies = max(1, min(8, -(-256 * 2**20 // wbytes)))
        qs = []
        for c in range(copies):
            wf = torch.randn(N, K, generator=g, device=dev) * 0.02
            if fmt == "fp8":
                codes, s_ = S.quantize_fp8(wf)
                qs.append({"fmt": "fp8", "w": codes, "s": s_.reshape(1), "N": N, "K": K})
            else:
                codes, sc, s2 = S.quantize_nvfp4(wf)
                qs.append({"fmt": "nvfp4", "w": codes, "sc": sc, "s": s2.reshape(1), "N": N, "K": K})
            del wf
        x = torch.randn(2, K, generator=g, device=dev).to(torch.bfloat16)
        cpu_q.append(({k_: (v_.cpu().numpy() if torch.is_tensor(v_) else v_) for k_, v_ in qs[0].items()},
                      x[0].float().cpu().numpy()))
        for M in (1, 2):
            with torch.cuda.stream(st):
                for q in qs:
                    D.gemv(q, x[0]) if M == 1 else D.gemv_mb(q, x[:M])
                gr = torch.cuda.CUDAGraph()
                reps = 4 * copies
                with torch.cuda.graph(gr, stream=st):
                    for r in range(reps):
                        q = qs[r % copies]
                        D.gemv(q, x[0]) if M == 1 else D.gemv_mb(q, x[:M])
                for _ in range(3):
                    gr.replay()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(st)
                for _ in range(10):
                    gr.replay()
                e1.record(st)
                e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (10 * reps)
            launches += 10 * reps
            b = wbytes + M * K * 2 + M * N * 4
            r_ = {"fmt": fmt, "N": N, "K": K, "M": M, "us": round(us, 3), "GB/s": round(b / us / 1e3, 1),
                  "frac": round(b / us / 1e3 / hbm, 4)}
            if M == 1:
                # end to end through dense_q.gemv: x from pinned host memory, y back to pinned host memory
                hx = x[0].cpu().pin_memory()
                dxx = torch.empty_like(x[0])
                with torch.cuda.stream(st):
                    y0 = D.gemv(qs[0], x[0])
                    hy = torch.empty(y0.shape, dtype=y0.dtype).pin_memory()
                    for _ in range(3):
                        dxx.copy_(hx, non_blocking=True)
                        hy.copy_(D.gemv(qs[0], dxx), non_blocking=True)
                    e2 = torch.cuda.Event(enable_timing=True)
                    e3 = torch.cuda.Event(enable_timing=True)
                    e2.record(st)
                    for r in range(reps):
                        dxx.copy_(hx, non_blocking=True)
                        hy.copy_(D.gemv(qs[r % copies], dxx), non_blocking=True)
                    e3.record(st)
                    e3.synchronize()
                r_["e2e_us"] = round(e2.elapsed_time(e3) * 1e3 / reps, 3)
                r_["h2d"] = int(hx.numel() * hx.element_size())
                r_["d2h"] = int(hy.numel() * hy.element_size())
            res.append(r_)
        del qs
        torch.cuda.empty_cache()
    tot_us = sum(r["us"] for r in res if r["M"] == 1)
    one = [r for r in res if r["M"] == 1]
    cpu_us = None if args.no_cpu_baseline else dense_cpu_reference(cpu_q)
    tot_b = sum((r["N"] * r["K"] if r["fmt"] == "fp8" else r["N"] * r["K"] * 9 // 16) for r in res if r["M"] == 1)
    line = {"metric": DENSE_METRIC, "value": round(tot_us, 3), "unit": "us (sum of shapes)",
            "n_gpus": 1, "steps": 10, "warmup": 3, "ms_per_step": round(tot_us / 1e3, 6), "scaling": "weak",
            "vs_baseline": None,
            "higher_is_better": False, "dtype": "fp8/nvfp4xbf16->f32", "data": "synthetic",
            "config": {"workload": "config2: dense_q GEMV sweep", "shapes": [list(s_) for s_ in DENSE_SHAPES],
                       "l2": "weight copies rotated beyond L2"},
            "roofline": {"bound": "hbm", "achieved": round(tot_b / tot_us / 1e3, 1), "peak": hbm, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(tot_b / tot_us / 1e3 / hbm, 4)},
            "per_shape": res,
            "e2e": {"value": round(sum(r["e2e_us"] for r in one), 3), "unit": "us (sum of shapes)",
                    "h2d_bytes_per_step": sum(r["h2d"] for r in one), "d2h_bytes_per_step": sum(r["d2h"] for r in one)},
            "gpu_launches": launches}
    if cpu_us is not None and all(c is not None for c in cpu_us):
        line["cpu_baseline"] = {"value": round(sum(cpu_us), 1), "unit": "us (sum of shapes)", "cores": 1, "kind": "port",
                                "sample": "each bs=1 shape once: oracle dequantize + matrix-vector product (fp64)"}
    print(json.dumps(line), flush=True)


PREFILL_FLOP_PER_PAIR = 2 * (2688 * 1024 + 1024 * 2688)   # up + down MACs x 2 = 11,010,048
PREFILL_METRIC = "MoE prefill tokens/s (one routed-expert layer, top-22 of 512)"


def prefill_cpu_reference(block_of, s2, ids, w, X, budget_s=15.0, threads=0, max_experts=48, return_out=False):
    """The reference's prompt path for T > 64 (nem_super.py:342-346) on the host cores: per expert hit,
    block_deq of its orig-layout block (the oracle's C restatement of qmoe_ns.py:407-412, fp32), then
    relu(F.linear(x, up))^2 and F.linear(h, down) on the expert's tokens in fp32 torch with all host threads,
    weighted and index-added into the output. A bounded sample: experts spread evenly over the ones hit (at
    most max_experts, or what the time budget allows), their times scaled to all experts hit.
    block_of(e) -> expert e's block as a numpy u8 array (fetched before its timing starts); s2 [ne, 2],
    ids [T, k] (-1 = none), w [T, k], X [T, 1024] (numpy). Returns (tokens/s, threads, sample text), and the
    output [T, 1024] of the sampled experts with return_out (all of them when the sample covers every expert)."""
    import numpy as np
    import torch
    import torch.nn.functional as F
    from oracle import oracle as O
    n = threads or host_cores()
    torch.set_num_threads(n)
    ids = np.asarray(ids)
    T = ids.shape[0]
    uniq = np.unique(ids[ids >= 0])
    pick = uniq[np.linspace(0, len(uniq) - 1, min(max_experts, len(uniq))).round().astype(int)]
    Xf = torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32))
    wf = np.asarray(w, np.float32)
    out = torch.zeros(T, 1024)
    times = []
    t_all = time.perf_counter()
    for e in pick:
        blk = block_of(int(e))
        tok, pos = np.nonzero(ids == e)
        t0 = time.perf_counter()
        u, d = O.block_deq(blk, s2[e])
        hh = torch.relu(F.linear(Xf[tok], torch.from_numpy(u))) ** 2
        yd = F.linear(hh, torch.from_numpy(d)) * torch.from_numpy(wf[tok, pos])[:, None]
        out.index_add_(0, torch.from_numpy(tok), yd)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    total_s = float(np.mean(times)) * len(uniq)
    res = (T / total_s, n, (f"{len(times)} of the {len(uniq)} experts hit (spread over the ids, with their tokens), "
                            f"mean {np.mean(times) * 1e3:.1f} ms/expert scaled to all {len(uniq)}"))
    return res + (out.numpy(),) if return_out else res


def tensor_peak():
    """NVFP4 dense tensor peak (TFLOP/s) and its description: 4 x the measured sustained cuBLAS bf16 rate."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpk = json.load(f)
        return 4.0 * float(tpk.get("bf16_tflops_sustained", tpk.get("bf16_tflops"))), \
            "NVFP4 dense = 4 x measured cuBLAS bf16 (sustained)"
    except Exception:
        return 4.0 * 1400.0, "NVFP4 dense = 4 x fallback bf16 (sustained 1.4 PF)"


def prefill_record(args, T, layout_T=False, steps=None, warmup=None, cpu=True, e2e=True):
    """the prompt path, one MoE layer of 512 synthetic NVFP4 experts (orig layout, the one
    the reference's moe_pairs reads, or the T layout, whose down halves the call converts first: 2 more kernels;
    1.585 GB resident in HBM), T tokens drawn as in config 0 and routed top-22 by the synthetic router; one step =
    one qmoe_prefill_grouped call: routing sort, x as NVFP4 planes (per token, then per pair), up GEMM + ReLU^2
    (block-scaled NVFP4 tcgen05), h as NVFP4 planes, down GEMM, combine - 10 kernels. value: tokens/s from CUDA
    events around K calls (inputs resident in HBM); e2e: the same call with the token block and routing copied
    from pinned host memory and the output copied back, every step. roofline: the whole call against the slower
    of the HBM bound (weights of the experts hit + activations) and the NVFP4 tensor bound (true FLOPs at 4x the
    measured dense bf16 rate, the FP4:bf16 ratio of the tensor cores); `pipe_flop` counts the MMA work actually
    issued (three activation planes). Returns the record (a dict)."""
    import torch
    import qmoe_ns as Q
    import qmoe_synth as S
    steps = args.steps if steps is None else steps
    warmup = max(3, args.warmup if warmup is None else warmup)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    hbm, peak_kind = peaks()
    tflops, tkind = tensor_peak()
    store, s2, m_hats, routers, _ = build_store(torch, S, dev, 1, seed=303, layout_T=layout_T)
    s2l = s2[0].contiguous()
    g = S.seeded(404, dev)
    X = S.tokens(T, m_hats[0], g, dev)
    ids, w = S.route(X, *routers[0])
    ids = ids.to(torch.int32).contiguous()
    w = w.float().contiguous()
    uniq = int(torch.unique(ids).numel())
    out = torch.empty(T, S.LAT, device=dev)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for _ in range(warmup):
            Q.moe_prefill(store, ids, w, s2l, X, layout_T=layout_T, out=out)
        st.synchronize()
        if Q.prefill_status() != 0:
            raise RuntimeError("prefill kernels reported a device-side error")
        clk = Clocks(0)
        clk.start()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            Q.moe_prefill(store, ids, w, s2l, X, layout_T=layout_T, out=out)
        e1.record(st)
        e1.synchronize()
        clocks = clk.stop()
        ms = e0.elapsed_time(e1) / steps
        ms_e2e, ee = None, max(5, steps // 2)
        if e2e:
            # every step: the prompt's tokens and routing from pinned host memory to the device, the call, and its
            # output back to pinned host memory. Prompts are independent, so as in a serving loop the copies run on
            # an upload and a download stream beside the calls: step i+1's upload and step i-1's download overlap
            # step i's call (double-buffered, each buffer reused only after the step that last used it is done).
            hx = X.cpu().pin_memory()
            hid = ids.cpu().pin_memory()
            hw = w.cpu().pin_memory()
            hout = [torch.empty(T, S.LAT, dtype=torch.float32).pin_memory() for _ in range(2)]
            dx = [torch.empty_like(X) for _ in range(2)]
            did = [torch.empty_like(ids) for _ in range(2)]
            dw = [torch.empty_like(w) for _ in range(2)]
            dout = [torch.empty_like(out) for _ in range(2)]
            us, ds = torch.cuda.Stream(), torch.cuda.Stream()
            up = [torch.cuda.Event() for _ in range(2)]
            done = [torch.cuda.Event() for _ in range(2)]
            down = [torch.cuda.Event() for _ in range(2)]
            e2 = torch.cuda.Event(enable_timing=True)
            e3 = torch.cuda.Event(enable_timing=True)
            e2.record(st)
            us.wait_event(e2)
            for i in range(ee):
                b = i & 1
                if i >= 2:
                    us.wait_event(done[b])      # step i-2 has read this input set
                with torch.cuda.stream(us):
                    dx[b].copy_(hx, non_blocking=True)
                    did[b].copy_(hid, non_blocking=True)
                    dw[b].copy_(hw, non_blocking=True)
                    up[b].record(us)
                st.wait_event(up[b])
                if i >= 2:
                    st.wait_event(down[b])      # step i-2's output has left this buffer
                Q.moe_prefill(store, did[b], dw[b], s2l, dx[b], layout_T=layout_T, out=dout[b])
                done[b].record(st)
                ds.wait_event(done[b])
                with torch.cuda.stream(ds):
                    hout[b].copy_(dout[b], non_blocking=True)
                    down[b].record(ds)
            st.wait_stream(us)
            st.wait_stream(ds)
            e3.record(st)
            e3.synchronize()
            ms_e2e = e2.elapsed_time(e3) / ee
            assert torch.equal(hout[(ee - 1) & 1], out.cpu())   # the last output back equals the device run's
    flop = T * K * PREFILL_FLOP_PER_PAIR
    wbytes = uniq * S.BLOCK
    act_bytes = T * S.LAT * 2 + T * S.LAT * 4 + T * K * 8
    t_hbm = (wbytes + act_bytes) / (hbm * 1e6)      # ms
    t_tc = flop / (tflops * 1e9)                    # ms
    if t_hbm >= t_tc:
        roof = {"bound": "hbm", "achieved": round((wbytes + act_bytes) / ms / 1e6, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(t_hbm / ms, 4), "peak_kind": f"{peak_kind} (HBM copy)"}
    else:
        roof = {"bound": "tensor", "achieved": round(flop / ms / 1e9, 1), "peak": tflops, "unit": "TFLOP/s",
                "frac": round(t_tc / ms, 4), "peak_kind": tkind}
    roof["traffic"] = None
    roof["algorithmic"] = {"flop": flop, "weight_bytes": wbytes, "activation_bytes": act_bytes,
                           "t_hbm_ms": round(t_hbm, 4), "t_tensor_ms": round(t_tc, 4),
                           "pipe_flop": 3 * flop, "pipe_tflops": round(3 * flop / ms / 1e9, 1)}
    rec = {"metric": PREFILL_METRIC, "value": round(T / ms * 1e3, 1), "unit": "tokens/s", "steps": steps,
           "warmup": warmup, "ms_per_step": round(ms, 5),
           "dtype": "nvfp4 weights x 3 nvfp4 activation planes -> f32 (tcgen05 kind::mxf4nvf4 block16)",
           "config": {"workload": f"config3: prefill T={T}", "T": T, "top_k": K, "experts": NE,
                      "unique_experts": uniq, "layout": "T" if layout_T else "orig",
                      "l2": "weights (1.585 GB) exceed L2"},
           "roofline": roof, "clocks": clocks, "gpu_launches": (12 if layout_T else 10) * steps}
    if ms_e2e is not None:
        rec["e2e"] = {"value": round(T / ms_e2e * 1e3, 1), "unit": "tokens/s",
                      "h2d_bytes_per_step": int(X.numel() * 2 + ids.numel() * 4 + w.numel() * 4),
                      "d2h_bytes_per_step": int(out.numel() * 4),
                      "copies": "every step: its tokens and routing up from pinned host memory, its output back; "
                                "on upload and download streams beside the calls (independent prompts, double-buffered)"}
    if cpu and not args.no_cpu_baseline:
        from oracle import oracle as O
        sh = s2l.cpu().numpy()

        def block_of(e):   # the orig-layout block (the reference's prompt path converts T blocks first)
            b = store[e].cpu().numpy()
            return O.from_T(b) if layout_T else b
        v, n, sample = prefill_cpu_reference(block_of, sh, ids.cpu().numpy(), w.cpu().numpy(),
                                             X.float().cpu().numpy(), budget_s=10.0)
        rec["cpu_baseline"] = {"value": round(v, 1), "unit": "tokens/s", "cores": n, "kind": "port", "sample": sample}
    del store
    torch.cuda.empty_cache()
    return rec


def run_decode_step(args):
    """--workload decode_step: the whole decode-step MoE block of every layer, one token through all layers in
    order as one CUDA graph (decode_step.DecodeGraph over decode_step.MoELayer: the router over the 4096-wide
    hidden state, the bf16 latent projections 4096 -> 1024 and 1024 -> 4096 as in the reference
    (nem_super.py:358-392), the 512 routed NVFP4 experts of config 1's store, the NVFP4 shared expert 2688 x 4096
    / 4096 x 2688), each layer's output feeding the next. value: us/token over K tokens rotating over 64 (inputs
    resident in HBM); the routed bytes are counted from the live groups and neurons each layer recorded for the
    tokens; the dense bytes are the layer weights. Synthetic weights: the live fractions follow from random
    projections, not config 1's recipe, and are reported."""
    import numpy as np
    import torch
    import decode_step as DS
    import expert_store as ES
    import qmoe_synth as S
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    L, H, SI = args.layers, 4096, 2688
    store, s2, _, _, _ = build_store(torch, S, dev, L, seed=1000, layout_T=True)
    est = ES.ExpertStore.from_tensors(store, s2, "T")
    g = S.seeded(616, dev)

    def nvfp4(n, k):
        codes, sc, s2_ = S.quantize_nvfp4(torch.randn(n, k, generator=g, device=dev) * 0.02)
        return {"fmt": "nvfp4", "w": codes, "sc": sc, "s": s2_.float().reshape(1), "N": n, "K": k}

    layers, dense_bytes = [], 0
    for m in range(L):
        gate = (torch.randn(NE, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        bias = torch.randn(NE, generator=g, device=dev) * 0.01
        fc1 = (torch.randn(S.LAT, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        fc2 = (torch.randn(H, S.LAT, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        layers.append(DS.MoELayer(m, est, gate, bias, fc1, fc2, nvfp4(SI, H), nvfp4(H, SI)))
        dense_bytes += 2 * (gate.numel() + fc1.numel() + fc2.numel()) + 2 * (SI * H // 2 + SI * H // 16)
    graph = DS.DecodeGraph(layers, H, device=dev)
    xs = torch.randn(N_TOK, H, generator=g, device=dev).to(torch.bfloat16)
    for i in range(max(3, args.warmup)):
        graph.replay(xs[i % N_TOK])
    torch.cuda.synchronize()
    clk = Clocks(0)
    clk.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()   # a profiler started with collection off (ncu --profile-from-start off) begins here
    e0.record()
    for i in range(args.steps):
        graph.replay(xs[(args.warmup + i) % N_TOK])
    e1.record()
    e1.synchronize()
    torch.cuda.profiler.stop()
    clocks = clk.stop()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    routed, live = [], []
    for t in range(4):   # the bytes the routed experts read for a few tokens, from what each layer recorded
        graph.replay(xs[t])
        torch.cuda.synchronize()
        b = n = 0
        for lay in layers:
            ex = lay.experts
            b += K * S.O_DW + 1024 * int(ex.gcnt.sum()) + 512 * int((ex.h > 0).sum())   # O_DW = the up half (UPB)
            n += int((ex.h > 0).sum())
        routed.append(b)
        live.append(n / (L * K * S.INTER))
    bytes_per_token = float(np.mean(routed)) + dense_bytes
    hbm, peak_kind = peaks()
    gbs = bytes_per_token / (us * 1e-6) / 1e9
    line = {"metric": "MoE decode-step us/token (whole MoE block: router, latent projections, routed and shared "
                      "experts, 40 layers, bs=1)", "value": round(us, 3), "unit": "us/token", "n_gpus": 1,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(us / 1e3, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4/bf16 -> f32",
            "data": "synthetic",
            "config": {"workload": "decode step: whole MoE block per layer, one CUDA graph per token", "layers": L,
                       "hidden": H, "experts": NE, "top_k": K, "tokens_rotated": N_TOK},
            "live_fraction": round(float(np.mean(live)), 4), "bytes_per_token": int(bytes_per_token),
            "dense_bytes_per_token": int(dense_bytes),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4), "traffic": None},
            "gpu_launches": 4 * L * args.steps,
            "gpu_launches_note": "libqmoe_b200 kernels (layer, finish, two shared-expert GEMVs per layer); torch's "
                                 "router, top-k and bf16 linears are not counted",
            "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_prefill(args):
    """--workload prefill: the prefill record of --prefill-t tokens as the line."""
    rec = prefill_record(args, args.prefill_t, layout_T=args.prefill_layout == "T")
    line = dict(rec)
    line.update({"n_gpus": 1, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "data": "synthetic"})
    print(json.dumps(line), flush=True)


def ep_init(world, rank, local):
    """The process group for expert parallelism (NCCL; a one-rank group when not launched by torchrun)."""
    import datetime
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local)
    if not dist.is_initialized():
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    return dev


EP_PHASES = ("pack", "dispatch", "experts", "return", "combine")


def ep_record(args, world, rank, local, batches=((64, "decode_batch"), (8192, "prefill")), layers=None):
    """expert parallelism. The 512 experts of every layer are sharded over the N ranks
    (expert e on rank e // (512 / N), orig layout, resident in HBM); each rank holds a batch of T tokens per
    layer. A step = `layers` MoE layers, each an ExpertParallelMoE forward: dispatch pack, NCCL all_to_all of the
    token blocks and routing, the local experts (block-scaled NVFP4 tcgen05 grouped GEMM), all_to_all of the
    partial outputs, rank-order combine. Per batch size: value = tokens of all ranks per second of max-over-ranks
    device time; `phases` = the per-step time of each phase, measured with CUDA events around the phases over one
    extra step (max over ranks), and `a2a_share` = the two exchanges' share of it. Every rank takes the same
    collective steps. Returns the record on rank 0 (None elsewhere)."""
    import torch
    import torch.distributed as dist
    import ep as EP
    import qmoe_ns as Q
    import qmoe_synth as S
    dev = ep_init(world, rank, local)
    L = args.layers if layers is None else layers
    el = NE // world
    g = S.seeded(1234 + rank, dev)
    # this rank's experts of every layer (generated on the device, orig layout)
    store = torch.empty(L * el, S.BLOCK, dtype=torch.uint8, device=dev)
    s2 = torch.empty(L, el, 2, dtype=torch.float32, device=dev)
    gl = S.seeded(99, dev)   # same m_hat / router on every rank
    m_hats = [S.unit_dir(gl, dev) for _ in range(L)]
    routers = [S.router(gl, dev) for _ in range(L)]
    p_l = S.layer_live_fractions(L) if L > 1 else [0.075]
    B = 16
    for m in range(L):
        for e0 in range(0, el, B):
            nb = min(B, el - e0)
            blk, s2b, _ = S.expert_blocks(nb, p_l[m], m_hats[m], g, dev)
            store[m * el + e0:m * el + e0 + nb].copy_(blk)
            s2[m, e0:e0 + nb] = s2b
            del blk
    moe = [EP.ExpertParallelMoE(store[m * el:(m + 1) * el], s2[m], n_experts=NE, layout_T=False) for m in range(L)]
    out = {"config": {"workload": f"config4: EP{world}, {L} layers", "layers": L, "experts_per_rank": el,
                      "parallelism": f"ep{world}", "exchange": "NCCL all_to_all, fixed T-row blocks"}}
    clocks = None
    for T, name in batches:
        steps = max(3, min(args.steps, 10 if T > 1024 else args.steps))
        warmup = 3
        gx = S.seeded(555 + rank, dev)
        X = [S.tokens(T, m_hats[m], gx, dev) for m in range(L)]
        R = [S.route(X[m], *routers[m]) for m in range(L)]

        def step(marks=None):
            for m in range(L):
                moe[m](X[m], R[m][0], R[m][1], marks=marks)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        if Q.prefill_status() != 0:
            raise RuntimeError("expert kernels reported a device-side error")
        clk = Clocks(local)
        if rank == 0:
            clk.start()
        dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        e1.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        c = clk.stop() if rank == 0 else None
        clocks = clocks or c
        ms = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms.item())
        # one more step with events between the phases of every layer
        marks = []
        step(marks)
        torch.cuda.synchronize()
        ph = {p: 0.0 for p in EP_PHASES}
        for i in range(len(marks)):
            name_i, ev = marks[i]
            if name_i in ph:
                ph[name_i] += marks[i - 1][1].elapsed_time(ev)
        pt = torch.tensor([ph[p] for p in EP_PHASES], device=dev)
        dist.all_reduce(pt, op=dist.ReduceOp.MAX)
        ph = {p: round(float(v), 4) for p, v in zip(EP_PHASES, pt.tolist())}
        tot = sum(ph.values())
        # e2e through the public module: host token blocks + routing in, host outputs back, every layer. The
        # layers' blocks here are independent, so the copies run on an upload and a download stream beside the
        # forwards: the next layer's upload and the previous layer's download overlap this layer's forward
        # (inputs double-buffered; each output is read back from its own tensor).
        hX = [x.cpu().pin_memory() for x in X]
        hI = [r[0].cpu().pin_memory() for r in R]
        hW = [r[1].cpu().pin_memory() for r in R]
        hO = torch.empty(L, T, S.LAT, dtype=torch.float32).pin_memory()
        dX = [torch.empty_like(X[0]) for _ in range(2)]
        dI = [torch.empty_like(R[0][0]) for _ in range(2)]
        dW = [torch.empty_like(R[0][1]) for _ in range(2)]
        us, ds = torch.cuda.Stream(), torch.cuda.Stream()
        up = [torch.cuda.Event() for _ in range(2)]
        used = [torch.cuda.Event() for _ in range(2)]
        ee = max(2, steps // 2)
        dist.barrier()
        torch.cuda.synchronize()
        cur = torch.cuda.current_stream()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record()
        us.wait_event(e2)
        q = 0
        for _ in range(ee):
            for m in range(L):
                b = q & 1
                if q >= 2:
                    us.wait_event(used[b])       # the forward two layers back has read this input set
                with torch.cuda.stream(us):
                    dX[b].copy_(hX[m], non_blocking=True)
                    dI[b].copy_(hI[m], non_blocking=True)
                    dW[b].copy_(hW[m], non_blocking=True)
                    up[b].record(us)
                cur.wait_event(up[b])
                y = moe[m](dX[b], dI[b], dW[b])
                used[b].record(cur)
                ds.wait_stream(cur)
                y.record_stream(ds)
                with torch.cuda.stream(ds):
                    hO[m].copy_(y, non_blocking=True)
                q += 1
        cur.wait_stream(us)
        cur.wait_stream(ds)
        e3.record()
        e3.synchronize()
        me = torch.tensor([e2.elapsed_time(e3) / ee], device=dev)
        dist.all_reduce(me, op=dist.ReduceOp.MAX)
        me = float(me.item())
        toks = T * world
        out[name] = {"tokens_per_rank": T, "value": round(toks / ms * 1e3, 1), "unit": "tokens/s",
                     "ms_per_step": round(ms, 4), "steps": steps, "warmup": warmup,
                     "phases_ms_per_step": ph, "a2a_share": round((ph["dispatch"] + ph["return"]) / tot, 4) if tot else None,
                     "e2e": {"value": round(toks / me * 1e3, 1), "unit": "tokens/s",
                             "h2d_bytes_per_step": int(L * T * (S.LAT * 2 + K * 12)),
                             "d2h_bytes_per_step": int(L * T * S.LAT * 4)},
                     "gpu_launches": L * steps * (2 + 10 + 1)}
        del X, R, hX, hI, hW, hO
    out["clocks"] = clocks
    del moe, store
    torch.cuda.empty_cache()
    dist.barrier()
    return out if rank == 0 else None


def run_ep(args):
    """--workload ep: the expert-parallel record of --ep-t tokens per rank as the line."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    rec = ep_record(args, world, rank, local, batches=((args.ep_t, "batch"),))
    if rank == 0:
        b = rec["batch"]
        line = {"metric": "MoE expert-parallel tokens/s (40-layer routed experts, top-22 of 512)", "value": b["value"],
                "unit": "tokens/s", "n_gpus": world, "steps": b["steps"], "warmup": b["warmup"],
                "ms_per_step": b["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "nvfp4 weights x 3 nvfp4 activation planes -> f32 (tcgen05 kind::mxf4nvf4 block16)",
                "data": "synthetic", "config": dict(rec["config"], tokens_per_rank=args.ep_t),
                "clocks": rec["clocks"], "e2e": b["e2e"], "gpu_launches": b["gpu_launches"],
                "phases_ms_per_step": b["phases_ms_per_step"], "a2a_share": b["a2a_share"]}
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "ep":
        return run_ep(args)
    if args.workload == "dense":
        return run_dense(args)
    if args.workload == "decode_step":
        return run_decode_step(args)
    import torch
    import torch.distributed as dist

    import _qmoe_lib as C
    import qmoe_synth as S
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    L = args.layers
    t0 = time.time()
    store, s2, m_hats, routers, p_l = build_store(torch, S, dev, L, seed=1000 + rank)
    T = make_tokens(torch, S, dev, store, s2, m_hats, routers, N_TOK, seed=2000 + rank)
    t_build = time.time() - t0

    step = DecodeStep(torch, dev, store, L)
    stream = torch.cuda.Stream(device=dev)
    # warm the library state (function attributes) outside capture
    with torch.cuda.stream(stream):
        step.launch(T["X"][0], T["SIDX"][0], T["TAB"][0], T["S2"][0], T["W"][0], stream.cuda_stream)
    stream.synchronize()
    # one graph per token of the stream (inputs resident in HBM)
    graphs = []
    for t in range(N_TOK):
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=stream):
            step.launch(T["X"][t], T["SIDX"][t], T["TAB"][t], T["S2"][t], T["W"][t], stream.cuda_stream)
        graphs.append(gph)
    torch.cuda.synchronize()

    # algorithmic bytes per token, averaged over the token stream
    tot_bytes, tot_groups, tot_neurons = 0, 0, 0
    for t in range(N_TOK):
        graphs[t].replay()
        torch.cuda.synchronize()
        b, gr, ne = algorithmic_bytes(torch, step, L)
        tot_bytes += b
        tot_groups += gr
        tot_neurons += ne
    bytes_per_token = tot_bytes / N_TOK
    live_frac = tot_neurons / (N_TOK * L * K * S.INTER)

    # ---- timed region: K steps of graph replay
    for i in range(args.warmup):
        graphs[i % N_TOK].replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = Clocks(local)
    clk.start()
    time.sleep(0.3)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for i in range(args.steps):
            graphs[(args.warmup + i) % N_TOK].replay()
        ev1.record(stream)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    clocks = clk.stop()
    t_max = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms = float(t_max.item())
    us_per_token = ms * 1e3 / (args.steps * world)
    us_per_token_rank = ms * 1e3 / args.steps

    # ---- the dominant kernel: decode_layer_kernel (up GEMV + ReLU^2 + live-neuron down GEMV of every expert,
    # one cluster per expert), with decode_finish_kernel (the 1024-row sum over experts) after it as its
    # programmatic dependent. The pair is timed as the layer it forms, from the CUDA events of the timed region
    # (device time per layer = step time / layers), against the layer's algorithmic bytes: every routed expert's
    # up half, the live neurons' dnT_w rows and live groups' dnT_s rows, x and y.
    layer_us = us_per_token_rank / L
    layer_bytes = bytes_per_token / L
    hbm, peak_kind = peaks()
    layer_gbs = layer_bytes / (layer_us * 1e-6) / 1e9

    # ---- e2e through the public path with host buffers, layer by layer as the model runs it: per layer the layer's
    # packed routed inputs (x, slot ids, block addresses, s2, weights) cross from pinned host memory
    # (qmoe_copy_async: a kernel chained after the previous layer's last kernel), the layer's qmoe_decode_groups
    # call runs, and its output y goes straight back into pinned host memory (the finish kernel's stores), each
    # layer after the previous one's output is back (layer m+1's input depends on layer m's output). The 40-layer
    # sequence is one CUDA graph; two pinned staging records alternate, each refilled on the host for the next
    # token once its last replay is done.
    REC = 2048 + K * (4 + 8 + 8 + 4)   # x bf16 | sidx i32 | tab i64 | s2 f32 x2 | coef f32
    offs = {"X": 0, "SIDX": 2048, "TAB": 2048 + 4 * K, "S2": 2048 + 12 * K, "W": 2048 + 20 * K}
    host_all = torch.empty(N_TOK, L, REC, dtype=torch.uint8)
    for k_, o_ in offs.items():
        src = T[k_].cpu().contiguous().view(torch.uint8).reshape(N_TOK, L, -1)
        host_all[:, :, o_:o_ + src.shape[2]] = src
    stage = [torch.empty(L, REC, dtype=torch.uint8).pin_memory() for _ in range(2)]
    rec_dev = torch.empty(L, REC, dtype=torch.uint8, device=dev)
    y_host = [torch.empty(L, S.LAT, dtype=torch.float32).pin_memory() for _ in range(2)]

    def view(k_, m, dt, n):
        return rec_dev[m, offs[k_]:offs[k_] + n * torch.tensor([], dtype=dt).element_size()].view(dt)

    fn = C.lib().qmoe_decode_groups
    cp = C.lib().qmoe_copy_async
    g_e2e = []
    for b in range(2):
        stage[b].copy_(host_all[0])
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=stream):
            for m in range(L):
                assert cp(rec_dev[m].data_ptr(), stage[b][m].data_ptr(), REC, stream.cuda_stream) == 0
                rc = fn(store.data_ptr(), store.stride(0), store.shape[0], view("SIDX", m, torch.int32, K).data_ptr(),
                        view("TAB", m, torch.int64, K).data_ptr(), view("S2", m, torch.float32, 2 * K).data_ptr(),
                        view("W", m, torch.float32, K).data_ptr(), view("X", m, torch.bfloat16, S.LAT).data_ptr(), 1, K,
                        step.h[m].data_ptr(), step.gidx[m].data_ptr(), step.gcnt[m].data_ptr(), step.part[m].data_ptr(),
                        y_host[b][m].data_ptr(), step.ws.data_ptr(), step.ws.numel(), stream.cuda_stream)
                assert rc == 0
        g_e2e.append(gph)
    done = [torch.cuda.Event(), torch.cuda.Event()]
    h2d = L * REC
    d2h = L * S.LAT * 4
    e_steps = max(20, args.steps // 2)

    def e2e_run(n, first):
        for i in range(n):
            b = i & 1
            done[b].synchronize()               # this staging record's last replay has finished reading it
            stage[b].copy_(host_all[(first + i) % N_TOK])
            g_e2e[b].replay()
            done[b].record(stream)

    with torch.cuda.stream(stream):
        e2e_run(args.warmup, 0)
        stream.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        e2e_run(e_steps, args.warmup)
        e1.record(stream)
        e1.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    # the last token's outputs came back and equal the device-resident path's for the same token
    ref_tok = (args.warmup + e_steps - 1) % N_TOK
    graphs[ref_tok].replay()
    torch.cuda.synchronize()
    e2e_ok = bool(torch.equal(y_host[(e_steps - 1) & 1], step.Y.cpu()))
    t_e2e = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(t_e2e, op=dist.ReduceOp.MAX)
    e2e_us = float(t_e2e.item()) * 1e3 / (e_steps * world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        s2_host = s2.cpu().numpy()
        cpu = cpu_baseline(store, s2_host, T, L, tok=args.warmup % N_TOK)

    line = None
    if rank == 0:
        step_gbs = bytes_per_token / (us_per_token_rank * 1e-6) / 1e9
        line = {
            "metric": METRIC, "value": round(us_per_token, 3), "unit": "us/token", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4xbf16->f32",
            "data": "synthetic",
            "config": decode_config(L, world),
            "live_fraction": round(live_frac, 4),
            "hbm_gbs_step": round(step_gbs, 1), "hbm_frac_step": round(step_gbs / hbm, 4),
            "bytes_per_token": int(bytes_per_token),
            "roofline": {"kernel": "decode_layer_kernel + decode_finish_kernel (one layer)", "bound": "hbm",
                         "achieved": round(layer_gbs, 1), "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(layer_gbs / hbm, 4),
                         "traffic": int(layer_bytes * LAYER_TRAFFIC_NCU["dram_bytes"] / LAYER_TRAFFIC_NCU["requested_bytes"]),
                         "traffic_source": "ncu single-launch capture of decode_layer_kernel: DRAM read + write "
                                           f"{LAYER_TRAFFIC_NCU['dram_bytes']} B against the "
                                           f"{LAYER_TRAFFIC_NCU['requested_bytes']} B its loads requested from L2 "
                                           "(a layer below the mean live fraction), the ratio scaled to this "
                                           "line's mean layer",
                         "bytes_per_launch": int(layer_bytes), "us_per_launch": round(layer_us, 3)},
            "e2e": {"value": round(e2e_us, 3), "unit": "us/token", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "copies": "per layer: its packed inputs read from pinned host memory by a chained copy kernel "
                             "(qmoe_copy_async), y written by the layer's finish kernel into pinned host memory",
                    "matches_device_path": e2e_ok},
            "gpu_launches": 2 * L * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "build_s": round(t_build, 1),
        }
    del graphs, g_e2e, step, store, T
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    # ---- sub-records: prefill (config 3, one GPU) and expert parallelism (config 4, every N)
    if world == 1 and not args.no_prefill:
        pre = prefill_record(args, 2048, steps=max(10, args.steps))
        pre["t64"] = prefill_record(args, 64, steps=max(10, args.steps), cpu=False, e2e=False)
        pre["t64"] = {k_: pre["t64"][k_] for k_ in ("value", "unit", "ms_per_step", "roofline")}
        line["prefill"] = pre
    if not args.no_ep:
        rec = ep_record(args, world, rank, local)
        if rank == 0:
            line["ep"] = rec
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
