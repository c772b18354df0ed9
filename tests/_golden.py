"""Loaders for the committed golden fixtures (produced by tests/golden/make_golden.py)."""
from __future__ import annotations

import os

import numpy as np

from oracle.model import Config

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
  return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def llm_case(tag):
  """(Config, weights dict, fixture) for one `llm_<tag>.npz` fixture."""
  z = load(f"llm_{tag}.npz")
  dim, nl, nh, nkv, ffn, vocab, hd = (int(v) for v in z["cfg"])
  cfg = Config(dim=dim, n_layers=nl, n_heads=nh, n_kv_heads=nkv, ffn_dim=ffn, vocab=vocab,
               head_dim=hd, rope_base=float(z["rope_base"]), norm_eps=float(z["norm_eps"]),
               qk_norm=bool(z["qk_norm"]))
  w = {"embed": z["embed"], "final_norm": z["final_norm"], "lm_head": z["lm_head"], "layers": []}
  for i in range(nl):
    pre = f"L{i}."
    w["layers"].append({k[len(pre):]: z[k] for k in z.files if k.startswith(pre)})
  return cfg, w, z
