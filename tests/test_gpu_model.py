"""The Llama3-style harness with Lighthouse layers trains on the GPU (small config)."""
import pytest
import torch


@pytest.mark.gpu
def test_small_model_trains(lh, cuda):
    from lighthouse_b200 import model as M
    args = M.ModelArgs(dim=256, n_layers=4, n_heads=2, n_kv_heads=2, hidden_dim=384, max_seq_len=4096,
                       lighthouse_topk=256, lighthouse_full_attn_layers=[0])
    torch.manual_seed(0)
    m = M.Transformer(args).to(cuda)
    m.init_weights(0)
    opt = torch.optim.AdamW(m.parameters(), lr=3e-3, fused=True)
    g = torch.Generator().manual_seed(1)
    # a repeating byte pattern is learnable: the loss must drop
    base = torch.randint(0, 256, (1, 64), generator=g)
    tokens = base.repeat(1, 4096 // 64 + 1)[:, :4097].to(cuda)
    losses = [M.train_step(m, opt, tokens).item() for _ in range(8)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0] - 0.5, losses
    assert lh._native.device_status() == 0
    assert sum(1 for layer in m.layers if layer.attention.lighthouse) == 3


def test_flavour_is_270m(lh):
    from lighthouse_b200 import model as M
    with torch.device("meta"):
        m = M.Transformer(M.ModelArgs())
    n = M.num_params(m)
    assert 2.5e8 < n < 3.0e8, n
