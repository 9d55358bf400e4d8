"""Host-side pieces of the config-5 LM (orthossm_b200.lm) that need no GPU:
the blocked restatement of the local-window attention against dense masked
attention, and the model's size at the spec's dimensions."""
import pytest
import torch
import torch.nn.functional as F

from orthossm_b200.lm import OrthoLMConfig, OrthoSSMLM, local_window_attention_blocked, n_params


@pytest.mark.parametrize("S,W", [(70, 16), (16, 16), (5, 16), (128, 32), (33, 8)])
def test_local_window_attention_matches_dense(S, W):
    torch.manual_seed(S * 100 + W)
    B, H, hd = 2, 3, 8
    q, k, v = (torch.randn(B, S, H, hd, dtype=torch.float64) for _ in range(3))
    i = torch.arange(S).view(S, 1)
    j = torch.arange(S).view(1, S)
    mask = (j <= i) & (j > i - W)
    ref = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                         attn_mask=mask).transpose(1, 2)
    assert (local_window_attention_blocked(q, k, v, W) - ref).abs().max().item() < 1e-12


def test_config5_size():
    m = OrthoSSMLM(OrthoLMConfig())
    assert m.lm_head.weight is m.embedding.weight
    assert n_params(m) == 24_282_672
