"""decode_step.route_tokens restates the router of the transformers NemotronH model (NemotronHTopkRouter.forward
tf:748-751 and NemotronHMoE.route_tokens_to_experts tf:697-720). On CPU, against the installed transformers'
own method bound to a stand-in module: identical expert ids and weights, for one expert group (the model's
setting) and for grouped routing with normalised weights."""
import types

import pytest
import torch

pytest.importorskip("transformers")


def _tf_route(x, gate_w, bias, top_k, scaling, n_group, topk_group, norm):
    from transformers.models.nemotron_h import modeling_nemotron_h as M
    fake = types.SimpleNamespace(
        gate=types.SimpleNamespace(e_score_correction_bias=bias), n_group=n_group, topk_group=topk_group,
        n_routed_experts=gate_w.shape[0], top_k=top_k, norm_topk_prob=norm, routed_scaling_factor=scaling)
    logits = torch.nn.functional.linear(x.to(torch.float32), gate_w.to(torch.float32))   # tf:748-751
    return M.NemotronHMoE.route_tokens_to_experts(fake, logits)


@pytest.mark.parametrize("n_group,topk_group,norm", [(1, 1, False), (8, 4, True), (4, 2, False)])
def test_route_tokens_matches_transformers(n_group, topk_group, norm):
    import decode_step as DS
    g = torch.Generator().manual_seed(11 + n_group)
    T, H, NE, K = 7, 256, 512, 22
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    gate = (torch.randn(NE, H, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.randn(NE, generator=g) * 0.01
    ids, w = DS.route_tokens(x, gate, bias, top_k=K, scaling=5.0, n_group=n_group, topk_group=topk_group,
                             norm_topk_prob=norm)
    rid, rw = _tf_route(x, gate, bias, K, 5.0, n_group, topk_group, norm)
    assert torch.equal(torch.sort(ids, dim=1).values, torch.sort(rid, dim=1).values)
    # same (id, weight) pairs
    o1, o2 = torch.argsort(ids, dim=1), torch.argsort(rid, dim=1)
    assert torch.equal(torch.gather(w, 1, o1), torch.gather(rw.to(w.dtype), 1, o2))
