"""Writes tests/golden/mamba2.npz: golden Mamba-2 decode steps from an independent
implementation, Hugging Face transformers 5.5.0's plain-torch Mamba2Mixer in float64 (run
here once; the fixture travels, this script does not need to).  Config-5-like ratios at a
small size: hidden 128, 4 heads x 64, state 32, 2 groups, conv width 4, A = -exp(U[0, 1]),
dt = softplus(in-projection + dt_bias), gated RMSNorm over the whole d_inner (the form
transformers implements).  Weights are rounded to float32 first so that the library's fp32
copies are the same numbers.  Six tokens for each of two sequences; the first goes through
transformers' chunked (SSD) prefill path, the next five through its recurrent decode path.

    python tests/golden/gen_mamba2.py
"""
import os

import numpy as np
import torch
from transformers import DynamicCache, Mamba2Config, Mamba2Model

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mamba2.npz")


def main():
    cfg = Mamba2Config(vocab_size=16, hidden_size=128, num_heads=4, head_dim=64, expand=2, state_size=32,
                       n_groups=2, conv_kernel=4, use_conv_bias=True, use_bias=False, num_hidden_layers=1,
                       layer_norm_epsilon=1e-5, chunk_size=8)
    torch.manual_seed(7)
    mix = Mamba2Model(cfg).eval().double().layers[0].mixer
    g = torch.Generator().manual_seed(8)
    with torch.no_grad():
        for name, t in mix.named_parameters():
            if name == "A_log":
                t.copy_(torch.rand(t.shape, generator=g, dtype=torch.float64))
            elif name == "dt_bias":
                t.copy_(torch.randn(t.shape, generator=g, dtype=torch.float64) * 0.5)
            else:
                t.copy_(torch.randn(t.shape, generator=g, dtype=torch.float64) * (0.08 if t.dim() > 1 else 0.5))
            t.copy_(t.float().double())                         # fp32-exact values
    cache = DynamicCache(config=cfg)
    T, B = 6, 2
    u = (torch.randn(T, B, 1, cfg.hidden_size, generator=g, dtype=torch.float64)).float().double()
    out = []
    with torch.no_grad():
        for t in range(T):
            out.append(mix(u[t], cache_params=cache)[:, 0].numpy())
    lay = cache.layers[0]
    np.savez_compressed(
        OUT, u=u[:, :, 0].numpy().astype(np.float32), out=np.stack(out),
        W_in=mix.in_proj.weight.detach().numpy().astype(np.float32), W_out=mix.out_proj.weight.detach().numpy().astype(np.float32),
        conv_w=mix.conv1d.weight[:, 0].detach().numpy().astype(np.float32), conv_b=mix.conv1d.bias.detach().numpy().astype(np.float32),
        A_log=mix.A_log.detach().numpy().astype(np.float32), dt_bias=mix.dt_bias.detach().numpy().astype(np.float32),
        D=mix.D.detach().numpy().astype(np.float32), norm_w=mix.norm.weight.detach().numpy().astype(np.float32),
        conv_state=lay.conv_states.numpy(), ssm_state=lay.recurrent_states.numpy(),
        dims=np.array([cfg.num_heads, cfg.head_dim, cfg.state_size, cfg.n_groups, cfg.conv_kernel]),
        eps=np.array([cfg.layer_norm_epsilon]))
    print("wrote", OUT)


if __name__ == "__main__":
    main()
