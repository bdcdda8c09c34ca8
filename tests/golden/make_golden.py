"""Generate the golden vectors by running the REFERENCE's own Python functions on CPU.

Run where a checkout of the reference is available, naming its root in NSREF:
    NSREF=<path to the reference checkout> python tests/golden/make_golden.py
Writes tests/golden/golden.npz and tests/golden/golden.json. The inputs are regenerated from seeds
by tests/golden/vectors.py, so only outputs are stored. Reference functions used:
  qmoe_ns.E2M1 (qmoe_ns.py:391), deq / block_deq (qmoe_ns.py:395-412), to_T / from_T
  (qmoe_ns.py:356-375), the live-group glue of moe_decode_groups (qmoe_ns.py:249-251, executed
  verbatim on the reference's h), the fp64 check of tests/kern_test.py:35-39, dense_q.dequant_rows
  (dense_q.py:179-188), and transformers' NemotronHMoE.route_tokens_to_experts (tf 5.5.0; the
  reference pins 5.9.0, whose routing function is called the same way).
"""
import hashlib
import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import vectors as V  # noqa: E402

REF = os.environ.get("NSREF")


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    if not REF or not os.path.isfile(os.path.join(REF, "qmoe_ns.py")):
        sys.exit("set NSREF to the root of the reference checkout (the directory holding qmoe_ns.py)")
    Q = _load("ref_qmoe_ns", os.path.join(REF, "qmoe_ns.py"))
    D = _load("ref_dense_q", os.path.join(REF, "dense_q.py"))
    out, meta = {}, {}

    # --- a1: decode tables
    out["e2m1"] = Q.E2M1.numpy().astype(np.float32)
    out["e4m3"] = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()

    # --- a11: deq, plus the SWAP negative control (tests/kern_test.py:42-47)
    b = V.rand_block(1)
    w = torch.from_numpy(b[V.O_UW:V.O_UW + 16 * 512].reshape(16, 512).copy())
    s = torch.from_numpy(b[V.O_US:V.O_US + 16 * 64].reshape(16, 64).copy())
    out["deq"] = Q.deq(w, s, 0.0123).numpy()
    Q.SWAP = True
    out["deq_swap"] = Q.deq(w, s, 0.0123).numpy()
    Q.SWAP = False

    # --- a10: to_T / from_T are byte permutations; hash the whole 3 MB outputs
    for seed in (2, 3):
        blk = torch.from_numpy(V.rand_bytes_block(seed))
        t = Q.to_T(blk)
        meta[f"to_T_{seed}"] = sha(t.numpy())
        meta[f"from_T_{seed}"] = sha(Q.from_T(blk).numpy())
        meta[f"roundtrip_{seed}"] = bool(torch.equal(Q.from_T(t), blk))
        # from_T_batch (qmoe_ns.py:378-387) on a batch of the T block
        g = t.clone().view(1, -1)
        Q.from_T_batch(g)
        meta[f"from_T_batch_{seed}"] = sha(g.numpy())

    # --- a2..a6: moe_decode in fp64 (tests/kern_test.py:35-39) + live groups (qmoe_ns.py:249-251)
    blocks, s2, coef, x = V.decode_case()
    K = len(blocks)
    xd = torch.from_numpy(x).double()
    ref = torch.zeros(1024, dtype=torch.float64)
    hs = []
    for j in range(K):
        u, d = Q.block_deq(torch.from_numpy(blocks[j]), torch.from_numpy(s2[j]))
        hh = torch.relu(u.double() @ xd) ** 2
        hs.append(hh)
        ref += float(coef[j]) * (d.double() @ hh)
    h = torch.stack(hs)
    out["decode_y"] = ref.numpy()
    out["decode_h"] = h.numpy()
    h_buf = h.float()
    glive = (h_buf[:K] > 0).view(K, 168, 16).any(-1)
    gcnt_buf = torch.empty(K, dtype=torch.int32)
    torch.sum(glive, dim=1, dtype=torch.int32, out=gcnt_buf[:K])
    gidx_buf = torch.empty(K, 168, dtype=torch.int32)
    gidx_buf[:K] = torch.sort(glive.to(torch.uint8), dim=1, descending=True, stable=True).indices.to(torch.int32)
    out["decode_gidx"] = gidx_buf.numpy()
    out["decode_gcnt"] = gcnt_buf.numpy()
    # the same blocks in the T layout must give the same y (layout is a pure permutation)
    meta["decode_T_blocks_sha"] = [sha(Q.to_T(torch.from_numpy(bk)).numpy()) for bk in blocks]

    # --- a7: moe_pairs in fp64 from block_deq (tests/pairs_test.py:34-46 pattern)
    blocks, pslot, ptok, s2p, coefp, X = V.pairs_case()
    res = []
    for p in range(len(pslot)):
        u, d = Q.block_deq(torch.from_numpy(blocks[pslot[p]]), torch.from_numpy(s2p[p]))
        hh = torch.relu(u.double() @ torch.from_numpy(X[ptok[p]]).double()) ** 2
        res.append(float(coefp[p]) * (d.double() @ hh))
    out["pairs_out"] = torch.stack(res).numpy()

    # --- a12..a15: dense dequant_rows (bf16 and fp32 outputs) and the fp64 GEMV
    for fmt, seed in (("fp8", 400), ("nvfp4", 401)):
        w, sc, s, xx = V.dense_case(fmt, seed)
        N = w.shape[0]
        Kd = w.shape[1] * (2 if fmt == "nvfp4" else 1)
        q = {"fmt": fmt, "w": torch.from_numpy(w), "s": torch.tensor([s], dtype=torch.float32), "N": N, "K": Kd}
        if sc is not None:
            q["sc"] = torch.from_numpy(sc)
        o16 = torch.empty(N, Kd, dtype=torch.bfloat16)
        D.dequant_rows(q, 0, N, o16)
        o32 = torch.empty(N, Kd, dtype=torch.float32)
        D.dequant_rows(q, 0, N, o32)
        out[f"dense_{fmt}_bf16"] = o16.view(torch.int16).numpy().view(np.uint16)
        out[f"dense_{fmt}_w32"] = o32.numpy()
        out[f"dense_{fmt}_y"] = (torch.from_numpy(xx).double() @ o32.double().t()).numpy()

    # --- a16: routing (tf:697-720), n_group=1, topk_group=1, top-22, x5.0, no normalisation
    from transformers.models.nemotron_h.modeling_nemotron_h import NemotronHMoE
    hh, gw, gb = V.route_case()
    logits = torch.nn.functional.linear(torch.from_numpy(hh), torch.from_numpy(gw))
    ns = types.SimpleNamespace(gate=types.SimpleNamespace(e_score_correction_bias=torch.from_numpy(gb)),
                               n_group=1, n_routed_experts=512, topk_group=1, top_k=22, norm_topk_prob=False,
                               routed_scaling_factor=5.0)
    ti, tw = NemotronHMoE.route_tokens_to_experts(ns, logits)
    order = torch.argsort(ti, dim=1)
    out["route_ids"] = torch.gather(ti, 1, order).numpy().astype(np.int64)
    out["route_w"] = torch.gather(tw, 1, order).numpy().astype(np.float32)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    meta["reference"] = "helgard-orlm/nemotron-super-8gb (qmoe_ns.py, dense_q.py) + transformers " + \
        __import__("transformers").__version__
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", sorted(out), sorted(meta))


if __name__ == "__main__":
    main()
