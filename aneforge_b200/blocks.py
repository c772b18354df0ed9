"""Decoder blocks as graph builders: the reference's registry-value form (`aneforge/llm.py:96-237`,
`PREFILL_MIXERS` / `DECODE_MIXERS` / `*_MLPS` values), written over this package's graph IR.

A graph builder returns graph Tensors; `compile` / `compile_multi` lower them, and `LlamaPrefill`
lowers registry entries of this form into its decode / prefill programs through the same lowering
(`llm.py`, graph-builder registry entries). The built-in "attention" / "swiglu" entries stay fused
plan emitters (the hot path); these builders are the general form - what a plugin written for the
reference registers - and the reference semantics the fused kernels are tested against.

Signatures follow the reference's registries:
  prefill mixer  f(x [S, D], w, cfg, ls, cos, sin) -> h            (`_attn_prefill`)
  decode mixer   f(x [1, D], w, cfg, ls, ctx, M) -> (h, [(state_out, state_in), ...])
  MLP            f(h, w, cfg, ls) -> h                             (prefill and decode alike)
with `w` the reference's layer dict, `ctx` the per-step decode inputs of `decode_inputs`.
"""
from __future__ import annotations

import numpy as np

from . import graph as G

F16 = np.float16

# per-step decode inputs a mixer may read from ctx: position one-hot and its complement over the
# cache rows, the additive mask, and the position's RoPE row (the reference's names and shapes)
DECODE_CTX = ("oh", "inv", "mask", "cosp", "sinp")


def decode_inputs(M: int, dh: int) -> dict:
  return {"oh": G.input((1, M, 1)), "inv": G.input((1, M, 1)), "mask": G.input((1, 1, M)),
          "cosp": G.input((1, dh)), "sinp": G.input((1, dh))}


def decode_values(pos: int, M: int, cos_t=None, sin_t=None) -> dict:
  """Host values of the per-step decode inputs at position `pos` (fp16)."""
  oh = np.zeros((1, M, 1), F16)
  oh[0, pos, 0] = 1
  v = {"oh": oh, "inv": (1 - oh).astype(F16), "mask": np.where(np.arange(M) <= pos, 0, -1e4).astype(F16).reshape(1, 1, M)}
  if cos_t is not None:
    v["cosp"] = np.asarray(cos_t[pos], F16)[None]
    v["sinp"] = np.asarray(sin_t[pos], F16)[None]
  return v


def rotate(x: G.Tensor, cos, sin) -> G.Tensor:
  """RoPE over the last axis, neox half-split: x * cos + [-x_hi, x_lo] * sin; cos / sin are fp16
  tables (baked) or graph Tensors (the decode step's row)."""
  dh, rank = x.shape[-1], len(x.shape)
  half = dh // 2
  size = list(x.shape[:-1]) + [half]
  lo = x.slice_by_size([0] * rank, size)
  hi = x.slice_by_size([0] * (rank - 1) + [half], size)
  c = cos if isinstance(cos, G.Tensor) else G.const(cos)
  s = sin if isinstance(sin, G.Tensor) else G.const(sin)
  return x * c + G.concat([hi * -1.0, lo], axis=rank - 1) * s


def _expand_matrix(kv: int, group: int) -> np.ndarray:
  """[kv * group, kv] 0/1: query head h reads kv head h // group."""
  return np.kron(np.eye(kv, dtype=F16), np.ones((group, 1), F16))


def expand_heads(k: G.Tensor, group: int) -> G.Tensor:
  """Grouped-query expansion of [KV, S, dh] (or [1, KV, S, dh]) to KV * group heads as a 0/1 matmul
  over the head axis - a `linear`, so under compress= the 0/1 matrix is encoded like any weight
  (the reference's `_repeat_kv3` / `_repeat_kv`, `aneforge/llm.py:108-116`, `:205-211`)."""
  if group == 1:
    return k
    # (nothing to expand)
  lead = len(k.shape) == 4
  kv, s, dh = k.shape[-3:]
  k3 = k.reshape(kv, s, dh) if lead else k
  out = k3.transpose([1, 2, 0]).linear(_expand_matrix(kv, group)).transpose([2, 0, 1])
  return out.reshape(1, kv * group, s, dh) if lead else out


def _norm_in(x: G.Tensor, w: dict, cfg, key: str) -> G.Tensor:
  if cfg.norm_type == "layer":
    return x.layer_norm(w[key + "_w"], w[key + "_b"], cfg.norm_eps)
  return x.rms_norm(w[key], cfg.norm_eps)


def _qkv(xn: G.Tensor, w: dict, cfg, ls, rows: int):
  H, KV, dh = cfg.n_heads, cfg.n_kv_heads, cfg.dh
  q = xn.linear(w["wq"], w.get("q_bias")).reshape(rows, H, dh)
  k = xn.linear(w["wk"], w.get("k_bias")).reshape(rows, KV, dh)
  v = xn.linear(w["wv"], w.get("v_bias")).reshape(rows, KV, dh)
  if ls.qk_norm:
    q = q.reshape(rows * H, dh).rms_norm(w["q_norm"], cfg.norm_eps).reshape(rows, H, dh)
    k = k.reshape(rows * KV, dh).rms_norm(w["k_norm"], cfg.norm_eps).reshape(rows, KV, dh)
  return q, k, v


def causal_attention(q: G.Tensor, k: G.Tensor, v: G.Tensor) -> G.Tensor:
  """softmax(q k^T / sqrt(dh) + causal mask) v over [1, H, S, dh]; masked scores get -1e4."""
  S, dh = q.shape[2], q.shape[3]
  mask = np.where(np.triu(np.ones((S, S), bool), 1), -1e4, 0).astype(F16)
  return ((q @ k.transpose([0, 1, 3, 2])) * (1.0 / dh ** 0.5) + G.const(mask)).softmax(-1) @ v


def attn_prefill_kv(x: G.Tensor, w: dict, cfg, ls, cos, sin):
  """Prompt attention (`aneforge/llm.py:149-169`): returns (x + o_proj(attention), (K, V)) with K
  (roped) and V in the decode cache layout [KV, S, dh]."""
  H, KV, dh, S = cfg.n_heads, cfg.n_kv_heads, cfg.dh, x.shape[0]
  q, k, v = _qkv(_norm_in(x, w, cfg, "attn_norm"), w, cfg, ls, S)
  q = q.transpose([1, 0, 2]).reshape(1, H, S, dh)
  k = k.transpose([1, 0, 2]).reshape(1, KV, S, dh)
  v = v.transpose([1, 0, 2]).reshape(1, KV, S, dh)
  if cfg.rope:
    q, k = rotate(q, cos, sin), rotate(k, cos, sin)
  kc, vc = k.reshape(KV, S, dh), v.reshape(KV, S, dh)
  a = causal_attention(q, expand_heads(k, H // KV), expand_heads(v, H // KV))
  a = a.reshape(H, S, dh).transpose([1, 0, 2]).reshape(S, H * dh)
  return x + a.linear(w["wo"], w.get("o_bias")), (kc, vc)


def attn_prefill(x: G.Tensor, w: dict, cfg, ls, cos, sin) -> G.Tensor:
  """Prompt attention without the cache outputs (`aneforge/llm.py:129-146`)."""
  return attn_prefill_kv(x, w, cfg, ls, cos, sin)[0]


def attn_decode(x: G.Tensor, w: dict, cfg, ls, ctx: dict, M: int):
  """One decode step against a resident cache (`aneforge/llm.py:214-237`): the mixer makes its own
  K / V state inputs [KV, M, dh], writes the step's k / v at the position through the one-hot
  (`K_out = K_in * inv + k * oh`) and attends over the masked cache. Returns (h, state pairs)."""
  H, KV, dh = cfg.n_heads, cfg.n_kv_heads, cfg.dh
  k_in, v_in = G.input((KV, M, dh)), G.input((KV, M, dh))
  q, k, v = _qkv(_norm_in(x, w, cfg, "attn_norm"), w, cfg, ls, 1)
  q, k, v = q.reshape(H, 1, dh), k.reshape(KV, 1, dh), v.reshape(KV, 1, dh)
  if cfg.rope:
    q, k = rotate(q, ctx["cosp"], ctx["sinp"]), rotate(k, ctx["cosp"], ctx["sinp"])
  k_out = k_in * ctx["inv"] + k * ctx["oh"]
  v_out = v_in * ctx["inv"] + v * ctx["oh"]
  kr, vr = expand_heads(k_out, H // KV), expand_heads(v_out, H // KV)
  p = ((q @ kr.transpose([0, 2, 1])) * (1.0 / dh ** 0.5) + ctx["mask"]).softmax(-1)
  a = (p @ vr).reshape(H, 1, dh).transpose([1, 0, 2]).reshape(1, H * dh)
  return x + a.linear(w["wo"], w.get("o_bias")), [(k_out, k_in), (v_out, v_in)]


def swiglu(h: G.Tensor, w: dict, cfg, ls) -> G.Tensor:
  """h + down(silu(gate(n)) * up(n)), n = rms_norm(h) (`aneforge/llm.py:171-175`)."""
  n = h.rms_norm(w["mlp_norm"], cfg.norm_eps)
  return h + (n.linear(w["wgate"]).silu() * n.linear(w["wup"])).linear(w["wdown"])


def gelu_tanh(x: G.Tensor) -> G.Tensor:
  """The tanh-form GELU, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), from primitive ops."""
  return (x * 0.5) * ((x + x.pow(3.0) * 0.044715) * float(np.sqrt(2.0 / np.pi))).tanh().adds(1.0)


def geglu(h: G.Tensor, w: dict, cfg, ls) -> G.Tensor:
  """h + down(gelu_tanh(gate(n)) * up(n)) (Gemma, `aneforge/llm.py:189-196`)."""
  n = h.rms_norm(w["mlp_norm"], cfg.norm_eps)
  return h + (gelu_tanh(n.linear(w["wgate"])) * n.linear(w["wup"])).linear(w["wdown"])


def gelu_mlp(h: G.Tensor, w: dict, cfg, ls) -> G.Tensor:
  """h + proj(gelu_tanh(fc(norm(h)))) (GPT-2, `aneforge/llm.py:178-183`)."""
  n = _norm_in(h, w, cfg, "mlp_norm")
  return h + gelu_tanh(n.linear(w["wfc"], w.get("fc_bias"))).linear(w["wproj"], w.get("proj_bias"))


def prefill_block(x: G.Tensor, w: dict, cfg, cos, sin, ls=None) -> G.Tensor:
  """One pre-norm block over a prompt: attention mixer then SwiGLU MLP."""
  from .llm import LayerSpec
  ls = ls or LayerSpec(qk_norm="q_norm" in w)
  return swiglu(attn_prefill(x, w, cfg, ls, cos, sin), w, cfg, ls)


def is_graph_builder(fn) -> bool:
  """True for a registry value written over graph Tensors (these builders, or a plugin's), False for
  a plan emitter (first parameter `pb`)."""
  import inspect
  try:
    params = list(inspect.signature(fn).parameters)
  except (TypeError, ValueError):
    return False
  return bool(params) and params[0] != "pb"
