"""Seeded random-init models in the reference weight layout, generated on the device.

The benchmark configurations have no checkpoints: their weights are N(0, 0.02), unit norms (the
shape of the reference's `tests/_helpers.py:make_random_llama_model`, with the benchmark's 0.02).
Generating them on the GPU keeps an 8B or 72B model off the host, and the layer list is lazy: each
layer is regenerated from its own seed when read and dropped afterwards, so the fp16 weights of
the whole model never exist at once - only the packed copy the loader keeps. The same seed gives
the same weights on the same device type, which is how tests rebuild a layer for the oracle.
"""
from __future__ import annotations


class LazyLayers:
  """The model's layer list; layer i is generated on access from seed * 1000 + i."""

  def __init__(self, cfg, device, seed, qkv_bias=False, moe=False, std=0.02):
    self.cfg, self.device, self.seed, self.qkv_bias, self.moe, self.std = cfg, device, seed, qkv_bias, moe, std

  def __len__(self):
    return self.cfg.n_layers

  def __getitem__(self, i):
    import torch
    if not 0 <= i < len(self):
      raise IndexError(i)
    cfg, dev = self.cfg, self.device
    g = torch.Generator(device=dev)
    g.manual_seed(self.seed * 1000 + i)
    R = lambda *s: (torch.randn(*s, generator=g, device=dev, dtype=torch.float32) * self.std).half()
    D, dh = cfg.dim, cfg.dh
    lw = {"wq": R(cfg.n_heads * dh, D), "wk": R(cfg.n_kv_heads * dh, D), "wv": R(cfg.n_kv_heads * dh, D),
          "wo": R(D, cfg.n_heads * dh), "attn_norm": torch.ones(D, device=dev), "mlp_norm": torch.ones(D, device=dev)}
    if self.moe:
      E, F = cfg.extra["n_experts"], cfg.ffn_dim
      lw.update(router=R(E, D), wgate_exps=R(E, F, D), wup_exps=R(E, F, D), wdown_exps=R(E, F, D))
    else:
      lw.update(wgate=R(cfg.ffn_dim, D), wup=R(cfg.ffn_dim, D), wdown=R(D, cfg.ffn_dim))
    if self.qkv_bias:
      lw.update(q_bias=R(cfg.n_heads * dh), k_bias=R(cfg.n_kv_heads * dh), v_bias=R(cfg.n_kv_heads * dh))
    return lw

  def __iter__(self):
    return (self[i] for i in range(len(self)))


def make_weights(cfg, device, seed=0, qkv_bias=False, moe=False, std=0.02):
  """Seeded N(0, std) fp16 weights on `device` in the reference dict layout (layers lazy)."""
  import torch
  g = torch.Generator(device=device)
  g.manual_seed(seed)
  R = lambda *s: (torch.randn(*s, generator=g, device=device, dtype=torch.float32) * std).half()
  D = cfg.dim
  return {"embed": R(cfg.vocab, D), "lm_head": R(cfg.vocab, D), "final_norm": torch.ones(D, device=device),
          "layers": LazyLayers(cfg, device, seed, qkv_bias, moe, std)}
