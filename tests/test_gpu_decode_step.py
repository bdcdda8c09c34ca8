"""The whole decode-step MoE layer on the device (nemotron-super-8gb_b200/decode_step.py), on synthetic
Nemotron-H weights: router 512 x hidden (bf16 + correction bias), fc1/fc2 latent projections in FP8, the
shared expert in NVFP4, 512 routed NVFP4 experts per layer (config 0 recipe) resident in an ExpertStore
(T layout). Checks:
* the layer output is within rel-L2 1e-2 (the bar for layer outputs against the fp32 dequantized path) of
  a reference built from torch dequantization and the fp64 expert oracle, with the same bf16 roundings
  between modules as the model (tf:722-737);
* the eager forward performs no host synchronisation (torch sync-debug mode "error");
* a 2-layer step recorded as one CUDA graph and replayed for two different tokens equals the eager run."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
H, LAT, SI, NE, K, NL = 2048, 1024, 2688, 512, 22, 2
E2M1 = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=torch.float32)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def deq_torch(q):
    """Independent torch dequantization of a dense_q dict (FP8: w*s; NVFP4: v*(sc*s2), dense_q.py:170-196)."""
    if q["fmt"] == "fp8":
        return q["w"].view(torch.float8_e4m3fn).float() * q["s"]
    w = q["w"]
    lut = E2M1.to(w.device)
    v = torch.stack([lut[(w & 15).long()], lut[(w >> 4).long()]], -1).reshape(q["N"], q["K"])
    sc = q["sc"].view(torch.float8_e4m3fn).float() * q["s"]
    return (v.view(q["N"], q["K"] // 16, 16) * sc[..., None]).reshape(q["N"], q["K"])


@pytest.fixture(scope="module")
def model():
    import expert_store as ES
    import qmoe_ns as Q
    import qmoe_synth as S
    import decode_step as DS
    g = S.seeded(515, DEV)
    blocks = torch.empty(NL * NE, Q.BLOCK, dtype=torch.uint8, device=DEV)
    s2 = torch.empty(NL, NE, 2, device=DEV)
    for m in range(NL):
        m_hat = S.unit_dir(g, DEV)
        for e0 in range(0, NE, 32):
            blk, s2b, _ = S.expert_blocks(32, 0.075, m_hat, g, DEV)
            blocks[m * NE + e0:m * NE + e0 + 32].copy_(blk)
            s2[m, e0:e0 + 32] = s2b
    orig = blocks.cpu().numpy()
    for m in range(NL):
        Q.to_T_batch(blocks[m * NE:(m + 1) * NE])
    store = ES.ExpertStore.from_tensors(blocks, s2, "T")

    def fp8(n, k):
        codes, s = S.quantize_fp8(torch.randn(n, k, generator=g, device=DEV) * 0.02)
        return {"fmt": "fp8", "w": codes, "s": s.float(), "N": n, "K": k}

    def nvfp4(n, k):
        codes, sc, s2_ = S.quantize_nvfp4(torch.randn(n, k, generator=g, device=DEV) * 0.02)
        return {"fmt": "nvfp4", "w": codes, "sc": sc, "s": s2_.float().reshape(1), "N": n, "K": k}

    layers = []
    for m in range(NL):
        gate = (torch.randn(NE, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
        bias = torch.randn(NE, generator=g, device=DEV) * 0.01
        layers.append(DS.MoELayer(m, store, gate, bias, fp8(LAT, H), fp8(H, LAT), nvfp4(SI, H), nvfp4(H, SI)))
    torch.cuda.synchronize()
    return dict(layers=layers, orig=orig, s2=s2.cpu().numpy(), g=g)


def reference_layer(layer, m, x, orig, s2):
    """fp32 torch + fp64 oracle path, bf16 between modules as in the model."""
    import decode_step as DS
    ids, w = DS.route_tokens(x, layer.gate_w, layer.bias)
    lat = (x.float() @ deq_torch(layer.fc1).t()).to(torch.bfloat16)
    idn = ids[0].cpu().numpy()
    y, _, _ = O.moe_decode([orig[m * NE + int(e)] for e in idn], s2[m][idn], w[0].float().cpu().numpy(),
                           lat[0].float().cpu().numpy())
    y = torch.from_numpy(y).float().to(DEV).view(1, -1).to(torch.bfloat16)
    out = (y.float() @ deq_torch(layer.fc2).t()).to(torch.bfloat16)
    u = torch.relu((x.float() @ deq_torch(layer.shared_up).t()).to(torch.bfloat16))
    sh = ((u * u).float() @ deq_torch(layer.shared_down).t()).to(torch.bfloat16)
    return out + sh


def test_layer_matches_fp32_path_without_host_sync(model):
    x = torch.randn(1, H, generator=model["g"], device=DEV).to(torch.bfloat16)
    layer = model["layers"][1]
    layer(x)                                   # first call creates the per-stream workspaces
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        y = layer(x)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    ref = reference_layer(layer, 1, x, model["orig"], model["s2"])
    assert y.shape == (1, H) and y.dtype == torch.bfloat16
    assert rel_l2(y.float().cpu().numpy(), ref.float().cpu().numpy()) < 1e-2


def test_step_graph_equals_eager(model):
    import decode_step as DS
    layers = model["layers"]
    graph = DS.DecodeGraph(layers, H)
    for seed in (1, 2):
        gx = torch.Generator(device=DEV)
        gx.manual_seed(seed)
        x = torch.randn(1, H, generator=gx, device=DEV).to(torch.bfloat16)
        h = x
        for layer in layers:
            h = layer(h)
        got = graph.replay(x).clone()
        torch.cuda.synchronize()
        assert rel_l2(got.float().cpu().numpy(), h.float().cpu().numpy()) < 1e-6


def test_fused_routing_matches_torch_routing(model):
    """qmoe_route_decode (one token: sigmoid, bias, top-22, weights and the store lookup in one kernel) against
    the torch routing (tf:697-720, 748-751) on the same fp32 logits: the same 22 experts with bit-identical
    weights, in order of decreasing choice; store rows, block addresses and s2 rows are those of the chosen
    experts. The torch routing stays the reference and the path for grouped or batched routing."""
    import decode_step as DS
    for m, layer in enumerate(model["layers"]):
        assert layer.fused
        st, ex = layer.experts.store, layer.experts
        for t in range(8):
            x = torch.randn(1, H, generator=model["g"], device=DEV).to(torch.bfloat16)
            ids_t, w_t = DS.route_tokens(x, layer.gate_w, layer.bias)
            ids, coef, sidx, tab, s2 = (a.clone() for a in layer.route_decode(x))
            ref = dict(zip(ids_t[0].tolist(), w_t[0].tolist()))
            got = dict(zip(ids.tolist(), coef.tolist()))
            assert set(got) == set(ref) and len(ids.unique()) == K
            assert all(got[e] == ref[e] for e in ref)                      # bit-identical weights
            choice = torch.nn.functional.linear(x.float(), layer.gate_w)[0].sigmoid() + layer.bias
            assert torch.all(choice[ids][:-1] >= choice[ids][1:])          # decreasing choice
            assert torch.equal(sidx, st.slot_index(ex.i, ids))
            assert torch.equal(tab, st.block_addresses(sidx))
            assert torch.equal(s2, st.s2[ex.i][ids])


def test_fused_shared_expert_is_bit_identical(model):
    """The shared expert through dq_gemv_nvfp4_bf16 (up projection with its squared ReLU, down projection with
    the add onto the routed output) equals the unfused torch sequence (qlinear, relu, square, qlinear, add)
    bit for bit, for the whole layer."""
    layer = model["layers"][0]
    for t in range(3):
        x = torch.randn(1, H, generator=model["g"], device=DEV).to(torch.bfloat16)
        fused = layer(x).clone()
        layer._fused_shared = lambda *a: False
        try:
            plain = layer(x).clone()
        finally:
            del layer._fused_shared
        assert torch.equal(fused, plain)


def test_bf16_projection_layer_is_bit_identical(model):
    """A layer whose latent projections are plain bf16 weights (as the reference's fc1 / fc2_latent_proj): the
    one-token path (fc1 on the side stream, fc2 reading y rounded to bf16 on load, the add in fc2's epilogue)
    equals the plain composition (bf16 GEMVs, y.to(bf16), the unfused shared expert, the add) bit for bit."""
    import decode_step as DS
    base = model["layers"][1]
    g = model["g"]
    fc1 = (torch.randn(LAT, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    fc2 = (torch.randn(H, LAT, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    layer = DS.MoELayer(1, base.experts.store, base.gate_w, base.bias, fc1, fc2, base.shared_up, base.shared_down)
    for t in range(3):
        x = torch.randn(1, H, generator=g, device=DEV).to(torch.bfloat16)
        fused = layer(x).clone()
        layer._fused_shared = lambda *a: False
        try:
            plain = layer(x).clone()
        finally:
            del layer._fused_shared
        assert torch.equal(fused, plain)
