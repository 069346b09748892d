"""C-JEPA object-slot predictor and its losses (CPU)."""
import torch

from drivedit_b200.models.causal_jepa import (CausalJEPALoss, CausalJEPAPredictor, SlotAttention,
                                              get_minimal_causal_jepa_config)


def test_slot_attention_shapes_and_competition():
    torch.manual_seed(0)
    sa = SlotAttention(num_slots=5, slot_dim=32, input_dim=16, num_iterations=2, hidden_dim=64)
    slots, attn = sa(torch.randn(3, 20, 16))
    assert slots.shape == (3, 5, 32) and attn.shape == (3, 5, 20)
    assert torch.allclose(attn.sum(1), torch.ones(3, 20), atol=1e-4)  # softmax over slots


def test_cjepa_forward_loss_backward_and_counterfactual():
    torch.manual_seed(0)
    cfg = get_minimal_causal_jepa_config()
    cfg.input_dim = 64
    m = CausalJEPAPredictor(cfg)
    feats = torch.randn(2, 4, 10, 64)
    out = m(feats)
    assert out["slots"].shape == (2, 4, 16, 128)
    assert out["predicted_slots"].shape == (2, cfg.prediction_horizon, 16, 128)
    assert out["object_mask_indices"].shape == (2, cfg.max_objects_masked)
    mi = out["object_mask_indices"]
    assert torch.equal(out["masked_slots"][0, :, mi[0, 0]], m.mask_token[0].expand(4, -1))
    losses = CausalJEPALoss(cfg)(out)
    assert {"slot_prediction", "trajectory", "contrastive", "total"} <= set(losses)
    losses["total"].backward()
    assert m.slot_encoder.slot_attention.to_k.weight.grad is not None
    cf = m.predict_counterfactual(feats, torch.tensor([[0, 1], [2, 3]]))
    assert cf["causal_effect"].shape == (2,)
    l2 = CausalJEPALoss(cfg)({**out, **cf})
    assert "counterfactual" in l2
