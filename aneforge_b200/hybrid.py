"""Qwen3.5 / Qwen3-Next hybrid decoders (reference `aneforge/qwen35.py`): a per-layer plan mixing
gated-DeltaNet linear-attention layers and gated full-attention layers, both registered as decode
mixers in the graph-builder form, so the runner lowers them into its decode program with their
states (the DeltaNet conv window and recurrent matrix, the attention K / V cache) resident on the
device.

Gated DeltaNet, one token (the recurrence of `Qwen3_5GatedDeltaNet` in transformers):
  mixed = W_qkv x (q | k | v channels), z = W_z x, beta = sigmoid(W_b x), a = W_a x
  conv window [CD, K] = (previous K - 1 inputs | mixed); c = silu(sum_k window * conv1d); the
  window's last K - 1 columns are the next conv state
  q, k (per key head) -> value heads, L2-normalised (q also scaled by dk^-1/2)
  g = exp(-exp(A_log) * softplus(a + dt_bias)) per value head
  S' = g S;  S_new = S' + k^T ((v - k S') beta);  o = q S_new
  out = out_proj(rmsnorm(o) * silu(z)), added to the residual.
Gated attention: q_proj yields the query and an output gate per head; QK-norm, partial RoPE, the
cache written at the position, GQA softmax attention, output times sigmoid(gate), o_proj.

`adapt` maps a Hugging Face Qwen3.5 text checkpoint (its (1 + w) RMSNorm weights baked, A_log
stored as -exp(A_log)); `load_gguf` reads the `qwen35` GGUF architecture."""
from __future__ import annotations

import numpy as np

from . import graph as G
from . import llm

F16, F32 = np.float16, np.float32


def _rotate_partial(x: G.Tensor, cosp, sinp, rd: int, interleaved: bool) -> G.Tensor:
  """RoPE over the first `rd` of the last axis (cos 1 / sin 0 past it in the step's row): the
  neox half split (i with i + rd/2) or GPT-J adjacent pairs."""
  dh, rank = x.shape[-1], len(x.shape)
  rd = rd or dh
  if interleaved:
    # adjacent pairs (2p, 2p + 1): a constant 0/+-1 matrix, applied as an fp16 matmul
    P = np.zeros((dh, dh), F32)
    for p in range(rd // 2):
      P[2 * p + 1, 2 * p] = -1.0
      P[2 * p, 2 * p + 1] = 1.0
    return x * cosp + (x @ G.const(P.astype(F16))) * sinp
  half = rd // 2
  lead = list(x.shape[:-1])
  lo = x.slice_by_size([0] * rank, lead + [half])
  hi = x.slice_by_size([0] * (rank - 1) + [half], lead + [half])
  parts = [hi * -1.0, lo]
  if rd < dh:
    parts.append(x.slice_by_size([0] * (rank - 1) + [rd], lead + [dh - rd]))     # times sin = 0
  return x * cosp + G.concat(parts, axis=rank - 1) * sinp


def gated_attention_decode(x: G.Tensor, w: dict, cfg, ls, ctx: dict, M: int):
  """Gated full attention for one token against a resident [KV, M, dh] cache (reference
  `aneforge/qwen35.py:28-51`). Returns (residual + o_proj(...), [(K_out, K_in), (V_out, V_in)])."""
  H, KV, dh, eps = cfg.n_heads, cfg.n_kv_heads, cfg.dh, cfg.norm_eps
  k_in, v_in = G.input((KV, M, dh)), G.input((KV, M, dh))
  xn = x.rms_norm(w["in_norm"], eps)
  qg = xn.linear(w["wq"]).reshape((H, 2 * dh))                 # per head: query | output gate
  q = qg.slice_by_size([0, 0], [H, dh]).rms_norm(w["q_norm"], eps)
  gate = qg.slice_by_size([0, dh], [H, dh]).reshape((1, H * dh))
  k = xn.linear(w["wk"]).reshape((KV, dh)).rms_norm(w["k_norm"], eps)
  v = xn.linear(w["wv"]).reshape((KV, 1, dh))
  q = _rotate_partial(q, ctx["cosp"], ctx["sinp"], cfg.rotary_dim, cfg.rope_interleaved).reshape((H, 1, dh))
  k = _rotate_partial(k, ctx["cosp"], ctx["sinp"], cfg.rotary_dim, cfg.rope_interleaved).reshape((KV, 1, dh))
  k_out = k_in * ctx["inv"] + k * ctx["oh"]
  v_out = v_in * ctx["inv"] + v * ctx["oh"]
  grouped = q.reshape((KV, H // KV, dh))                       # query heads of one kv head together
  p = ((grouped @ k_out.transpose([0, 2, 1])) * (1.0 / dh ** 0.5) + ctx["mask"]).softmax(-1)
  att = (p @ v_out).reshape((1, H * dh)) * gate.sigmoid()
  return x + att.linear(w["wo"]), [(k_out, k_in), (v_out, v_in)]


def _head_map(nk: int, nv: int, tiled: bool) -> np.ndarray:
  """[nv, nk] 0/1: value head h reads key head h // (nv / nk) (transformers), or h % nk (GGUF /
  llama.cpp, which repeats the key heads as a whole)."""
  g = nv // nk
  h = np.arange(nv)
  src = h % nk if tiled else h // g
  m = np.zeros((nv, nk), F16)
  m[h, src] = 1
  return m


def gated_deltanet_decode(x: G.Tensor, w: dict, cfg, ls, ctx: dict, M: int):
  """Gated DeltaNet for one token (reference `aneforge/qwen35.py:54-88`), its own states: the conv
  window [CD, K - 1] and the recurrent matrix [nv, dk, dv]. `ctx` / `M` are unused (no positions).
  Returns (residual + out_proj(...), [(conv_out, conv_in), (state_out, state_in)])."""
  e, eps = cfg.extra, cfg.norm_eps
  nk, nv, dk, dv, K = int(e["nk"]), int(e["nv"]), int(e["dk"]), int(e["dv"]), int(e["conv_k"])
  kd, vd = nk * dk, nv * dv
  CD = 2 * kd + vd
  conv_in, s_in = G.input((CD, K - 1)), G.input((nv, dk, dv))
  xn = x.rms_norm(w["in_norm"], eps)
  mixed = xn.linear(w["in_proj_qkv"]).reshape((CD, 1))
  z = xn.linear(w["in_proj_z"]).reshape((nv, dv))
  beta = xn.linear(w["in_proj_b"]).reshape((1, nv)).sigmoid().reshape((nv, 1, 1))
  a = xn.linear(w["in_proj_a"]).reshape((1, nv))
  window = G.concat([conv_in, mixed], axis=1)                 # [CD, K], oldest column first
  c = (window * G.const(np.asarray(w["conv1d"], F32))).sum([1]).reshape((1, CD)).silu()
  conv_out = window.slice_by_size([0, 1], [CD, K - 1])
  hm = G.const(_head_map(nk, nv, e.get("gqa_repeat") == "tile"))
  q = (hm @ c.slice_by_size([0, 0], [1, kd]).reshape((nk, dk))).l2_norm(-1, 1e-6) * float(dk ** -0.5)
  k = (hm @ c.slice_by_size([0, kd], [1, kd]).reshape((nk, dk))).l2_norm(-1, 1e-6)
  v = c.slice_by_size([0, 2 * kd], [1, vd]).reshape((nv, 1, dv))
  q, k = q.reshape((nv, 1, dk)), k.reshape((nv, 1, dk))
  decay = ((a + G.const(np.asarray(w["dt_bias"], F32))).softplus() * G.const(np.asarray(w["neg_exp_A"], F32))).exp()
  s_dec = s_in * decay.reshape((nv, 1, 1))
  delta = (v - k @ s_dec) * beta                               # [nv, 1, dv]
  s_out = s_dec + k.transpose([0, 2, 1]) @ delta               # rank-1 update per value head
  o = (q @ s_out).reshape((nv, dv)).rms_norm(w["ssm_norm"], eps) * z.silu()
  return x + o.reshape((1, vd)).linear(w["out_proj"]), [(conv_out, conv_in), (s_out, s_in)]


llm.DECODE_MIXERS["gated_deltanet"] = gated_deltanet_decode
llm.DECODE_MIXERS["gated_attention"] = gated_attention_decode


def _is_full_attention(c, n):
  kinds = getattr(c, "layer_types", None)
  if kinds:
    return [t == "full_attention" for t in kinds[:n]]
  every = int(getattr(c, "full_attention_interval", 4) or 4)
  return [(li + 1) % every == 0 for li in range(n)]


def adapt(c, sd: dict, prefix: str = ""):
  """(LlamaConfig, weights) of a Hugging Face Qwen3.5 / Qwen3-Next text checkpoint (reference
  `aneforge/qwen35.py:94-131`); `prefix` is the layers' key prefix ('model.language_model.' in the
  vision-language checkpoint). The (1 + w) RMSNorm weights are baked (the gated SSM norm is plain)
  and -exp(A_log) is stored, so the mixers read uniform weights."""
  n = int(c.num_hidden_layers)
  full = _is_full_attention(c, n)
  hd = int(getattr(c, "head_dim", 0) or 0)
  rp = getattr(c, "rope_parameters", None)
  prf = (rp.get("partial_rotary_factor") if isinstance(rp, dict) else None) or getattr(c, "partial_rotary_factor", 1.0)
  theta = (rp.get("rope_theta") if isinstance(rp, dict) else None) or getattr(c, "rope_theta", 1e4)
  cfg = llm.LlamaConfig(dim=int(c.hidden_size), n_layers=n, n_heads=int(c.num_attention_heads),
                        n_kv_heads=int(c.num_key_value_heads), ffn_dim=int(c.intermediate_size),
                        vocab=int(c.vocab_size), rope_base=float(theta), norm_eps=float(c.rms_norm_eps), head_dim=hd,
                        rotary_dim=int((hd or c.hidden_size // c.num_attention_heads) * float(prf)),
                        layers=[llm.LayerSpec(mixer="gated_attention" if f else "gated_deltanet") for f in full],
                        extra={"nk": int(c.linear_num_key_heads), "nv": int(c.linear_num_value_heads),
                               "dk": int(c.linear_key_head_dim), "dv": int(c.linear_value_head_dim),
                               "conv_k": int(c.linear_conv_kernel_dim)})
  get = lambda k: np.asarray(sd[prefix + k])
  one_plus = lambda k: (get(k).astype(F32) + 1.0)
  embed = get("embed_tokens.weight")
  w = {"embed": embed, "final_norm": one_plus("norm.weight"), "lm_head": np.asarray(sd.get("lm_head.weight", embed)),
       "layers": []}
  for li in range(n):
    p = f"layers.{li}."
    lw = {"in_norm": one_plus(p + "input_layernorm.weight"), "mlp_norm": one_plus(p + "post_attention_layernorm.weight"),
          "wgate": get(p + "mlp.gate_proj.weight"), "wup": get(p + "mlp.up_proj.weight"),
          "wdown": get(p + "mlp.down_proj.weight")}
    if full[li]:
      a = p + "self_attn."
      lw.update(wq=get(a + "q_proj.weight"), wk=get(a + "k_proj.weight"), wv=get(a + "v_proj.weight"),
                wo=get(a + "o_proj.weight"), q_norm=one_plus(a + "q_norm.weight"), k_norm=one_plus(a + "k_norm.weight"))
    else:
      d = p + "linear_attn."
      lw.update(in_proj_qkv=get(d + "in_proj_qkv.weight"), in_proj_z=get(d + "in_proj_z.weight"),
                in_proj_a=get(d + "in_proj_a.weight"), in_proj_b=get(d + "in_proj_b.weight"),
                conv1d=np.squeeze(get(d + "conv1d.weight")).astype(F32),
                neg_exp_A=-np.exp(get(d + "A_log").astype(F32)), dt_bias=get(d + "dt_bias").astype(F32),
                ssm_norm=get(d + "norm.weight"), out_proj=get(d + "out_proj.weight"))
    w["layers"].append(lw)
  return cfg, w
