"""LayerwiseModel.fused_projections: stacked q/k/v and gate/up weights whose
rows the HF modules then alias (CPU, the mock decoder)."""
import torch

from helpers import mock_model


def test_fused_projections_stack_and_alias():
    from cacheblend import LayerwiseModel
    model = mock_model()
    lw = LayerwiseModel.from_hf(model)
    ids = torch.randint(0, model.config.vocab_size, (1, 40), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        before = model(input_ids=ids).logits
        originals = [(l.self_attn.q_proj.weight.clone(), l.self_attn.k_proj.weight.clone(),
                      l.self_attn.v_proj.weight.clone(), l.mlp.gate_proj.weight.clone(),
                      l.mlp.up_proj.weight.clone()) for l in model.model.layers]
        for li, layer in enumerate(model.model.layers):
            w_qkv, w_gu = lw.fused_projections(li)
            q, k, v, g, u = originals[li]
            assert torch.equal(w_qkv, torch.cat([q, k, v])) and torch.equal(w_gu, torch.cat([g, u]))
            attn, mlp = layer.self_attn, layer.mlp
            # the modules' weights are row views of the stacked ones
            assert attn.k_proj.weight.data_ptr() == w_qkv[q.shape[0]:].data_ptr()
            assert mlp.up_proj.weight.data_ptr() == w_gu[g.shape[0]:].data_ptr()
            assert torch.equal(attn.v_proj.weight, v) and torch.equal(mlp.gate_proj.weight, g)
            assert lw.fused_projections(li)[0] is w_qkv               # built once
        after = model(input_ids=ids).logits
    assert torch.equal(before, after)
