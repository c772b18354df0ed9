"""Decoder numerics: numpy restatement of the reference's quantized Llama/Qwen/MoE prefill and
KV-cache decode (`aneforge/llm.py`, `aneforge/moe.py`) as the reference lowers it
(`aneforge/_compile.py`).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

Precision policy. The reference's graph runs with fp16 ports; its off-device numpy stand-in
computes everything else in fp32. This oracle has two modes:

  * precision="fp32"   - fp16 at ports (program inputs/outputs, resident KV state), fp32 for every
                         internal node. Pinned against golden vectors from the reference's own
                         `LlamaPrefill` driving a numpy interpreter of its graph IR.
  * precision="device" - the same, plus every activation operand of a matmul (`linear`,
                         `bmm_weight`, and the q/K/V operands of attention's `bmm`s) rounded to fp16
                         first, which is what the fp16 device operands of the B200 kernels (and of
                         the ANE) see. Attention probabilities stay fp32. The GPU parity tests use
                         this mode.

Reference quirks restated here (each cites where the reference does it):
  * RMSNorm is `x / max(||x||_2, f16(sqrt(D*eps))) * f16(gamma*sqrt(D))` (`_compile.py:738-755`).
  * The attention scale is the fp16-rounded `1/sqrt(dh)` of a `muls` (`llm.py:234`, `_compile.py:334-346`).
  * GQA expansion is a 0/1 `linear` that is itself encoded by `compress` (`llm.py:205-211`,
    `_compile.py:375-379`): under int8 each expanded K/V row is scaled by 127*f16(1/127).
  * The mask is an additive -1e4 (`llm.py:124`, `:587`); masked keys contribute exactly 0.
  * RoPE tables are float64 -> fp16 (`llm.py:76-94`); rotation `x*cos + cat(-x2, x1)*sin` (`llm.py:96-105`).
  * The lm_head is the host fp32 matmul of the fp16 hidden row (`llm.py:349-355`).
  * MoE top-k peels the row max k times, lowest index on exact ties (`moe.py:21-37`); the
    `bmm_weight` down projection is encoded with ONE per-expert row (`_compile.py:393-399`).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import quant
from .quant import encode_weight

F16, F32 = np.float16, np.float32


# ----------------------------------------------------------------------------- config / tables

@dataclass
class Config:
  """The fields of reference `LlamaConfig` (`aneforge/llm.py:45-59`) the path needs."""
  dim: int; n_layers: int; n_heads: int; n_kv_heads: int; ffn_dim: int; vocab: int
  rope_base: float = 10000.0; norm_eps: float = 1e-5; head_dim: int = 0
  rotary_dim: int = 0; rope_scaling: dict | None = None
  extra: dict = field(default_factory=dict)
  qk_norm: bool = False
  mlp: str = "swiglu"            # "swiglu", "geglu", "gelu_new" or "moe"
  norm_type: str = "rms"         # "rms" or "layer" (LayerNorm with bias, GPT-2)
  rope: bool = True              # False: learned positions (`wpe`) added to the embedding

  @property
  def dh(self) -> int:
    return self.head_dim or self.dim // self.n_heads


def llama3_rope_scale(inv, s):
  """Reference `aneforge/llm.py:62-73` (HF "llama3" inverse-frequency rescaling)."""
  factor, lo, hi = float(s["factor"]), float(s["low_freq_factor"]), float(s["high_freq_factor"])
  old = float(s["original_max_position_embeddings"])
  low_wl, high_wl = old / lo, old / hi
  wl = 2.0 * np.pi / inv
  scaled = np.where(wl > low_wl, inv / factor, inv)
  smooth = (old / wl - lo) / (hi - lo)
  smoothed = (1.0 - smooth) * scaled / factor + smooth * scaled
  return np.where((wl >= high_wl) & (wl <= low_wl), smoothed, scaled)


def rope_tables(seq: int, dh: int, base: float = 10000.0, rotary_dim: int = 0, scaling=None):
  """Neox half-split cos/sin tables [seq, dh], float64 math cast to fp16 (reference `llm.py:76-94`)."""
  rd = rotary_dim or dh
  inv = 1.0 / (base ** (np.arange(0, rd, 2) / rd))
  if scaling and scaling.get("rope_type") == "llama3":
    inv = llama3_rope_scale(inv, scaling)
  pos = np.arange(seq)[:, None] * inv[None, :]
  emb = np.concatenate([pos, pos], -1)
  c, s = np.cos(emb), np.sin(emb)
  if rd < dh:
    c = np.concatenate([c, np.ones((seq, dh - rd))], 1)
    s = np.concatenate([s, np.zeros((seq, dh - rd))], 1)
  return c.astype(F16), s.astype(F16)


def rms_consts(gamma: np.ndarray, eps: float):
  """The two constants the reference bakes for `rms_norm` (`_compile.py:738-748`):
  g_eff = f16(f32(gamma) * sqrt(D)) and floor = f16(sqrt(D * eps))."""
  D = int(np.asarray(gamma).shape[-1])
  g = (np.asarray(gamma).reshape(1, D).astype(F32) * float(np.sqrt(D))).astype(F16)
  floor = np.float16((D * float(eps)) ** 0.5)
  return g.reshape(D), floor


def rms_norm(x: np.ndarray, g_eff: np.ndarray, floor) -> np.ndarray:
  """`mul(real_div(x, maximum(reduce_l2_norm(x), floor)), g_eff)` over the last axis, fp32."""
  x = x.astype(F32)
  nrm = np.sqrt(np.sum(x * x, axis=-1, keepdims=True, dtype=F32)).astype(F32)
  sn = np.maximum(nrm, F32(floor))
  return ((x / sn) * g_eff.astype(F32)).astype(F32)


def layer_norm(x: np.ndarray, g: np.ndarray, b: np.ndarray, eps) -> np.ndarray:
  """Reference `_e_layer_norm` (`_compile.py:758-776`) in fp32: xc = x - mean(x),
  xc * rsqrt(mean(xc^2) + eps) * g + b, eps rounded to fp16 as the emitter bakes it."""
  x = x.astype(F32)
  xc = (x - x.mean(axis=-1, keepdims=True, dtype=F32)).astype(F32)
  var = (xc * xc).mean(axis=-1, keepdims=True, dtype=F32)
  rr = (F32(1.0) / np.sqrt(var + F32(np.float16(eps)))).astype(F32)
  return ((xc * rr) * np.asarray(g, F32) + np.asarray(b, F32)).astype(F32)


def norm_consts(w: dict, key: str, cfg) -> tuple:
  """An encoded norm: ("ln", gamma, beta, eps) for LayerNorm models, else the RMSNorm constants."""
  if cfg.norm_type == "layer":
    return ("ln", np.asarray(w[key + "_w"], F16), np.asarray(w[key + "_b"], F16), cfg.norm_eps)
  return rms_consts(w[key], cfg.norm_eps)


def apply_norm(x: np.ndarray, spec) -> np.ndarray:
  if len(spec) == 4 and isinstance(spec[0], str):
    return layer_norm(x, *spec[1:])
  return rms_norm(x, *spec)


def rope(x: np.ndarray, c: np.ndarray, s: np.ndarray) -> np.ndarray:
  """`x*cos + cat(-x2, x1)*sin` over the last axis (reference `llm.py:96-105`), fp32."""
  half = x.shape[-1] // 2
  rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
  return (x * c.astype(F32) + rot * s.astype(F32)).astype(F32)


def silu(x: np.ndarray) -> np.ndarray:
  return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
  m = x.max(axis=axis, keepdims=True)
  e = np.exp(x - m)
  return (e / e.sum(axis=axis, keepdims=True)).astype(F32)


# ----------------------------------------------------------------------------- the model

class Linear:
  """One encoded matmul weight [OUT, IN] (+ fp16 bias) with the device-order dequant: for int8
  the per-row scale multiplies the fp32 dot product."""

  def __init__(self, W, bias, compress, atol=0.05, block_size=32, allow_sparse=True, int8=None):
    self.enc = encode_weight(np.asarray(W), compress, atol, block_size, allow_int8=True,
                             allow_int4=True, allow_sparse=allow_sparse, int8=int8)
    self.bias = None if bias is None else np.asarray(bias, F32).astype(F16).astype(F32)
    if self.enc.kind == "int8":
      q, s = self.enc.parts
      self.qT = np.ascontiguousarray(q.astype(F32).T)
      self.s = s.astype(F32)
    else:
      self.WT = np.ascontiguousarray(self.enc.deq.reshape(self.enc.deq.shape[0], -1).T)

  @classmethod
  def from_codes(cls, q: np.ndarray, s: np.ndarray, bias=None) -> "Linear":
    """An int8 per-row Linear from codes [OUT, IN] and fp16 scales [OUT] already produced by the
    per-row quantizer (`quant.quantize_per_row`), skipping the encode step."""
    lin = cls.__new__(cls)
    lin.enc = quant.Encoded("int8", None, (np.asarray(q, np.int8), np.asarray(s, F16)))
    lin.bias = None if bias is None else np.asarray(bias, F32).astype(F16).astype(F32)
    lin.qT = np.ascontiguousarray(np.asarray(q).astype(F32).T)
    lin.s = np.asarray(s, F16).astype(F32)
    return lin

  def __call__(self, x: np.ndarray) -> np.ndarray:
    if self.enc.kind == "int8":
      y = (x @ self.qT) * self.s
    else:
      y = x @ self.WT
    if self.bias is not None:
      y = y + self.bias
    return y.astype(F32)


class OracleModel:
  """Reference-semantics decoder over a reference-layout weight dict (`aneforge/llm.py:636-654`:
  embed, final_norm, lm_head, layers[i] with wq/wk/wv/wo/wgate/wup/wdown/attn_norm/mlp_norm and the
  optional q/k/v/o biases and q/k norms; MoE layers carry router/wgate_exps/wup_exps/wdown_exps)."""

  def __init__(self, cfg: Config, weights: dict, compress: str | None = None,
               precision: str = "device", compress_atol: float = 0.05, block_size: int = 32,
               moe_compress: str | None = "same"):
    if precision not in ("fp32", "device"):
      raise ValueError(precision)
    self.cfg, self.w, self.compress, self.precision = cfg, weights, compress, precision
    # expert weights may use their own format (e.g. int4_g32 experts with int8 attention); the
    # reference has one compress= for the whole graph, which is the default here
    self.moe_compress = compress if moe_compress == "same" else moe_compress
    self.atol, self.bs = compress_atol, block_size
    H, KV, dh, D = cfg.n_heads, cfg.n_kv_heads, cfg.dh, cfg.dim
    self.g = H // KV
    self.scale16 = F32(np.float16(1.0 / dh ** 0.5))
    Mx = np.repeat(np.eye(KV, dtype=F16), self.g, axis=0)          # reference llm.py:209
    self.Mx = (encode_weight(Mx, compress, compress_atol, block_size).deq.astype(F32)
               if self.g > 1 else None)
    self.layers = [self._encode_layer(lw) for lw in weights["layers"]]
    self.final_norm = norm_consts(weights, "final_norm", cfg)
    self.wpe = weights.get("wpe")
    self.lmT = np.ascontiguousarray(np.asarray(weights["lm_head"]).T, F32)
    self.embed = weights["embed"]

  # -- encoding
  def _encode_layer(self, lw):
    cfg, c = self.cfg, self.compress
    L = {"wq": Linear(lw["wq"], lw.get("q_bias"), c, self.atol, self.bs),
         "wk": Linear(lw["wk"], lw.get("k_bias"), c, self.atol, self.bs),
         "wv": Linear(lw["wv"], lw.get("v_bias"), c, self.atol, self.bs),
         "wo": Linear(lw["wo"], lw.get("o_bias"), c, self.atol, self.bs)}
    L["attn_norm"] = norm_consts(lw, "attn_norm", cfg)
    L["mlp_norm"] = norm_consts(lw, "mlp_norm", cfg)
    if "q_norm" in lw:
      L["q_norm"] = rms_consts(lw["q_norm"], cfg.norm_eps)
      L["k_norm"] = rms_consts(lw["k_norm"], cfg.norm_eps)
    if "router" in lw:
      L["moe"] = self._encode_moe(lw)
    elif "wfc" in lw:                                              # GPT-2 GELU MLP, with biases
      L["wfc"] = Linear(lw["wfc"], lw.get("fc_bias"), c, self.atol, self.bs)
      L["wproj"] = Linear(lw["wproj"], lw.get("proj_bias"), c, self.atol, self.bs)
    else:
      L["wgate"] = Linear(lw["wgate"], None, c, self.atol, self.bs)
      L["wup"] = Linear(lw["wup"], None, c, self.atol, self.bs)
      L["wdown"] = Linear(lw["wdown"], None, c, self.atol, self.bs)
    return L

  def _encode_moe(self, lw):
    """Encodings exactly as `moe._moe` builds them (`aneforge/moe.py:40-63`): the router is a
    `linear`; gate/up are `linear`s over the expert-concatenated [g*ffn, dim] tiles of
    `_experts_gate` (tile = 65536 // ffn experts); down is one `bmm_weight` whose encoding sees
    [E, ffn*dim] (one row per expert)."""
    c = self.moe_compress
    E, ffn, dim = lw["wgate_exps"].shape
    gtile = max(1, min(E, 65536 // ffn))
    m = {"router": Linear(lw["router"], None, c, self.atol, self.bs), "E": E, "ffn": ffn}
    if "wgate_sh" in lw:
      # Qwen2-MoE's always-on shared expert and its sigmoid gate (`aneforge/moe.py:60-62`): plain
      # `linear`s, encoded by the graph's compress= like the router
      for key in ("wgate_sh", "wup_sh", "wdown_sh", "shared_gate"):
        m[key] = Linear(lw[key], None, self.compress, self.atol, self.bs)
    for key in ("wgate_exps", "wup_exps"):
      tiles = []
      for s0 in range(0, E, gtile):
        n = min(gtile, E - s0)
        tiles.append(Linear(lw[key][s0:s0 + n].reshape(n * ffn, dim), None, c, self.atol, self.bs))
      m[key] = (tiles, gtile)
    Wd = np.asarray(lw["wdown_exps"])
    m["router"] = Linear(lw["router"], None, self.compress, self.atol, self.bs)
    if c == "int4_g32":
      # this build's group-32 format groups along the contraction axis: each expert's down matrix is
      # quantized as [dim, ffn] (groups of 32 along ffn); no reference counterpart
      deq = [quant.dequant_g32_int4(*quant.quantize_g32_int4(np.ascontiguousarray(Wd[e].T))).T for e in range(E)]
      m["wdown"] = np.stack(deq).astype(F32)
      return m
    enc = encode_weight(Wd, c, self.atol, self.bs, allow_int8=True, allow_int4=True, allow_sparse=False)
    m["wdown"] = enc.deq.reshape(E, ffn, dim).astype(F32)
    return m

  # -- helpers
  def _mm_in(self, x):
    """The activation operand of a matmul: fp16-rounded in device mode."""
    return x.astype(F16).astype(F32) if self.precision == "device" else x.astype(F32)

  def _lin(self, L, x):
    return L(self._mm_in(x))

  def _expand(self, K):
    """`_repeat_kv3`: [KV, S, dh] -> [H, S, dh] via the encoded 0/1 matrix (identity when g == 1)."""
    if self.Mx is None:
      return K
    Kin = self._mm_in(K)
    return np.einsum("hk,ksd->hsd", self.Mx, Kin, dtype=F32).astype(F32)

  # -- blocks
  def _qkv(self, L, h, S):
    cfg = self.cfg
    H, KV, dh = cfg.n_heads, cfg.n_kv_heads, cfg.dh
    xn = apply_norm(h, L["attn_norm"])
    q = self._lin(L["wq"], xn).reshape(S, H, dh)
    k = self._lin(L["wk"], xn).reshape(S, KV, dh)
    v = self._lin(L["wv"], xn).reshape(S, KV, dh)
    if "q_norm" in L:
      q = rms_norm(q, *L["q_norm"]); k = rms_norm(k, *L["k_norm"])
    return q, k, v

  def _attend(self, q, Kr, Vr, n_valid):
    """q [H, Sq, dh]; Kr/Vr [H, Sk, dh]; n_valid(i) = number of visible keys for query row i."""
    sc = np.einsum("hqd,hkd->hqk", self._mm_in(q), self._mm_in(Kr), dtype=F32) * self.scale16
    Sq, Sk = sc.shape[1], sc.shape[2]
    mask = np.zeros((Sq, Sk), F32)
    for i in range(Sq):
      mask[i, n_valid(i):] = F32(np.float16(-1e4))
    p = softmax(sc + mask[None])
    # probabilities stay fp32: a flash-style kernel never materialises the normalised fp16 P
    return np.einsum("hqk,hkd->hqd", p, self._mm_in(Vr), dtype=F32).astype(F32)

  def _mlp(self, L, h):
    if "moe" in L:
      return self._moe(L["moe"], h)
    hn = apply_norm(h, L["mlp_norm"])
    act = silu(self._lin(L["wgate"], hn)) * self._lin(L["wup"], hn)
    return (h + self._lin(L["wdown"], act)).astype(F32)

  def decode_layer(self, L, h, Kc, Vc, pos):
    """One decode step of one layer (reference `_attn_decode` + MLP, `llm.py:214-237`).
    h [1, D] fp32; Kc/Vc [KV, M, dh] fp16 resident state, updated in place at `pos`."""
    cfg = self.cfg
    H, dh = cfg.n_heads, cfg.dh
    q, k, v = self._qkv(L, h, 1)
    q, k, v = q[0], k[0], v[0]                                     # [H, dh], [KV, dh]
    if cfg.rope:
      c, s = self.cos[pos], self.sin[pos]
      q = rope(q, c, s); k = rope(k, c, s)
    # Kout = Kin*inv + k*oh: fp32 internally, slot `pos` holds the unrounded k
    Kw = Kc[:, : pos + 1].astype(F32); Vw = Vc[:, : pos + 1].astype(F32)
    Kw[:, pos] = k; Vw[:, pos] = v
    Kc[:, pos] = k.astype(F16); Vc[:, pos] = v.astype(F16)
    a = self._attend(q[:, None, :], self._expand(Kw), self._expand(Vw), lambda i: pos + 1)
    h = h + self._lin(L["wo"], a.reshape(1, H * dh))
    return self._mlp(L, h)

  def decode_step(self, tok: int, pos: int, caches) -> np.ndarray:
    """Embedding gather -> all layers -> final norm; returns the fp16 hidden port [D]."""
    h = np.asarray(self.embed[tok])[None].astype(F16).astype(F32)
    if self.wpe is not None:
      h = (h + np.asarray(self.wpe[pos], F32)).astype(F32)
    for L, (Kc, Vc) in zip(self.layers, caches):
      h = self.decode_layer(L, h, Kc, Vc, pos)
    return apply_norm(h, self.final_norm).astype(F16)[0]

  def prefill_hidden(self, token_ids):
    """Batched prefill (reference `_prefiller`/`_attn_prefill_kv`, `llm.py:149-169`, `:489-519`).
    Returns (hidden [S, D] fp16 port, [(K [KV,S,dh] f16, V f16)] per layer)."""
    ids = np.asarray(token_ids)
    return self.causal_pass(np.asarray(self.embed[ids]), self.layers)

  def causal_pass(self, rows, layers):
    """The batched-prefill numerics over embedding rows [S, D] (fp16 port) through `layers`, an
    iterable of encoded layers (`_encode_layer` output, or `encoded_layer_from_codes`) consumed one
    at a time - a caller may build each layer on demand so that only one is in memory. Returns
    (hidden [S, D] fp16, [(K, V)] per layer). Causal attention over the rows is also the decode
    recurrence along the same tokens (teacher forcing): every matmul operand is rounded to fp16 in
    device mode either way, so a cached fp16 K/V row and the fresh fp32 one enter alike."""
    cfg = self.cfg
    H, KV, dh = cfg.n_heads, cfg.n_kv_heads, cfg.dh
    S = int(np.shape(rows)[0])
    self._tables(S)
    c, s = self.cos[:S], self.sin[:S]
    h = np.asarray(rows).astype(F16).astype(F32)
    if self.wpe is not None:                                       # learned positions 0..S-1, fp32 add
      h = (h + np.asarray(self.wpe[:S], F32)).astype(F32)
    kv = []
    for L in layers:
      q, k, v = self._qkv(L, h, S)
      q, k, v = q.transpose(1, 0, 2), k.transpose(1, 0, 2), v.transpose(1, 0, 2)   # [H, S, dh]
      if cfg.rope:
        q = rope(q, c, s); k = rope(k, c, s)
      kv.append((k.astype(F16), v.astype(F16)))
      a = self._attend(q, self._expand(k), self._expand(v), lambda i: i + 1)
      h = h + self._lin(L["wo"], a.transpose(1, 0, 2).reshape(S, H * dh))
      h = self._mlp(L, h)
    return apply_norm(h, self.final_norm).astype(F16), kv

  def encoded_layer_from_codes(self, codes: dict, norms: dict):
    """An encoded int8 layer from per-row codes: `codes` maps wq/wk/wv/wo/wgate/wup/wdown to
    (q, s) or (q, s, bias); `norms` maps attn_norm/mlp_norm (and q_norm/k_norm) to gamma."""
    L = {}
    for key, parts in codes.items():
      L[key] = Linear.from_codes(*parts)
    for key, gamma in norms.items():
      L[key] = rms_consts(gamma, self.cfg.norm_eps)
    return L

  def logits(self, hidden_row) -> np.ndarray:
    """Host fp32 lm_head (reference `llm.py:349-355`)."""
    return np.asarray(hidden_row, F32) @ self.lmT

  def _tables(self, M):
    cfg = self.cfg
    if getattr(self, "_M", -1) < M:
      self.cos, self.sin = rope_tables(M, cfg.dh, cfg.rope_base, cfg.rotary_dim, cfg.rope_scaling)
      self._M = M

  def new_caches(self, M):
    cfg = self.cfg
    return [(np.zeros((cfg.n_kv_heads, M, cfg.dh), F16), np.zeros((cfg.n_kv_heads, M, cfg.dh), F16))
            for _ in self.layers]

  @staticmethod
  def sample(logits, temperature, top_p, top_k):
    """Reference `LlamaPrefill._sample` (`llm.py:407-419`)."""
    if temperature <= 0.0:
      return int(np.argmax(logits))
    lg = logits.astype(np.float64) / temperature
    if top_k and 0 < top_k < lg.size:
      lg[lg < np.partition(lg, -top_k)[-top_k]] = -np.inf
    p = np.exp(lg - lg.max()); p /= p.sum()
    if 0.0 < top_p < 1.0:
      order = np.argsort(p)[::-1]; cum = np.cumsum(p[order])
      keep = order[:int(np.searchsorted(cum, top_p)) + 1]
      m = np.zeros_like(p); m[keep] = p[keep]; p = m / m.sum()
    return int(np.random.choice(p.size, p=p))

  def generate(self, token_ids, max_new_tokens=40, eos_id=None, max_len=None, temperature=0.0,
               top_p=1.0, top_k=0, batched_prefill=True, prefill_pad=None, return_logits=False):
    """Reference `LlamaPrefill.generate` control flow (`llm.py:560-633`), host lm_head."""
    prompt = [int(t) for t in token_ids]
    M = int(max_len or len(prompt) + max_new_tokens)
    eos = {int(eos_id)} if isinstance(eos_id, int) else {int(e) for e in (eos_id or ())}
    self._tables(M)
    caches = self.new_caches(M)
    out, all_logits = [], []
    if batched_prefill and len(prompt) > 1:
      real = len(prompt)
      seq = max(int(prefill_pad), real) if prefill_pad else real
      hid, kv = self.prefill_hidden(prompt + [0] * (seq - real))
      self._tables(M)
      for (Kc, Vc), (K, V) in zip(caches, kv):
        Kc[:, :real] = K[:, :real]; Vc[:, :real] = V[:, :real]
      lg = self.logits(hid[real - 1].astype(F32))
      all_logits.append(lg)
      cur = self.sample(lg, temperature, top_p, top_k); out.append(cur)
      if cur in eos:
        return (out, all_logits) if return_logits else out
      pos = real
    else:
      for p, tok in enumerate(prompt[:-1]):
        self.decode_step(tok, p, caches)
      cur, pos = prompt[-1], len(prompt) - 1
    while len(out) < max_new_tokens:
      if pos >= M - 1:
        break
      hid = self.decode_step(cur, pos, caches)
      lg = self.logits(hid.astype(F32))
      all_logits.append(lg)
      nxt = self.sample(lg, temperature, top_p, top_k)
      out.append(nxt)
      if nxt in eos:
        break
      cur, pos = nxt, pos + 1
    return (out, all_logits) if return_logits else out


# ----------------------------------------------------------------------------- MoE

def topk_gate(probs: np.ndarray, k: int) -> np.ndarray:
  """Reference `moe._topk_gate` (`aneforge/moe.py:21-37`): k rounds of row-max peel, lowest index
  on exact ties, exactly k experts per row; returns probs masked to the chosen experts."""
  T, E = probs.shape
  if not 1 <= k <= E <= 2049:
    raise ValueError(f"moe top-k: need 1 <= k <= E <= 2049; got k={k}, E={E}")
  rem = probs.astype(F32).copy()
  chosen = np.zeros((T, E), F32)
  ar = np.arange(E)
  for _ in range(k):
    hit = rem >= rem.max(axis=1, keepdims=True)
    first = np.where(hit, ar[None, :], 4096).min(axis=1, keepdims=True)
    pick = ar[None, :] == first
    chosen = np.where(pick, F32(1.0), chosen)
    rem = np.where(pick, F32(np.float16(-3.0e4)), rem)
  return (probs * chosen).astype(F32)


def _moe(self, m, h):
  """Reference `moe._moe` (`aneforge/moe.py:48-63`) for routed experts; dense over all E like the
  reference (non-selected experts carry weight exactly 0)."""
  cfg = self.cfg
  e = cfg.extra
  E, k = e["n_experts"], e["n_experts_per_tok"]
  ffn, T = m["ffn"], h.shape[0]
  L = self._cur_layer
  hn = apply_norm(h, L["mlp_norm"])
  probs = softmax(self._lin(m["router"], hn))
  gw = topk_gate(probs, k)
  if e.get("norm_topk_prob", True):
    gw = (gw / gw.sum(axis=1, keepdims=True)).astype(F32)
  def experts(key):
    tiles, g = m[key]
    parts = [self._lin(t, hn).reshape(T, -1, ffn) for t in tiles]
    return np.concatenate(parts, axis=1)                           # [T, E, ffn]
  act = silu(experts("wgate_exps")) * experts("wup_exps")
  out = np.einsum("tef,efd->etd", self._mm_in(act), m["wdown"], dtype=F32)   # [E, T, dim]
  comb = (out * gw.T[:, :, None]).sum(axis=0).astype(F32)
  if "wgate_sh" in m:
    sh_act = silu(self._lin(m["wgate_sh"], hn)) * self._lin(m["wup_sh"], hn)
    gate = (F32(1.0) / (F32(1.0) + np.exp(-self._lin(m["shared_gate"], hn)))).astype(F32)   # [T, 1]
    comb = (comb + self._lin(m["wdown_sh"], sh_act) * gate).astype(F32)
  return (h + comb).astype(F32)


def _mlp_with_moe(self, L, h):
  if "moe" in L:
    self._cur_layer = L
    return _moe(self, L["moe"], h)
  hn = apply_norm(h, L["mlp_norm"])
  if "wfc" in L:                                                   # GPT-2 (`aneforge/llm.py:178-183`)
    return (h + self._lin(L["wproj"], gelu_tanh(self._lin(L["wfc"], hn)))).astype(F32)
  g = self._lin(L["wgate"], hn)
  act = (gelu_tanh(g) if self.cfg.mlp == "geglu" else silu(g)) * self._lin(L["wup"], hn)
  return (h + self._lin(L["wdown"], act)).astype(F32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
  """The reference's GeGLU activation built from graph ops (`aneforge/llm.py:184-187`):
  (x * 0.5) * (tanh((x + x^3 * 0.044715) * sqrt(2/pi)) + 1), its scalar constants baked fp16 like
  every constant of the reference program."""
  c1 = F32(np.float16(0.044715))
  c2 = F32(np.float16(np.sqrt(2.0 / np.pi)))
  x = x.astype(F32)
  return ((x * F32(0.5)) * (np.tanh((x + (x ** 3) * c1) * c2) + F32(1.0))).astype(F32)


OracleModel._mlp = _mlp_with_moe


# ----------------------------------------------------------------------------- standalone pieces

def gemv_int8(x: np.ndarray, q: np.ndarray, s: np.ndarray, bias=None) -> np.ndarray:
  """Config-1 GEMV: y = x . (scale (.) W_q)^T, fp32 accumulation, fp16 out."""
  y = (x.astype(F32) @ q.astype(F32).T) * s.astype(F32)
  if bias is not None:
    y = y + np.asarray(bias, F16).astype(F32)
  return y.astype(F16)


def decoder_block_step(cfg: Config, lw: dict, h: np.ndarray, Kc, Vc, pos: int, compress="int8",
                       precision="device"):
  """Config-2 single decode step of one block, no final norm: returns fp16 hidden [1, D]."""
  w = {"layers": [lw], "final_norm": np.ones(cfg.dim, F32), "embed": np.zeros((1, cfg.dim), F16),
       "lm_head": np.zeros((1, cfg.dim), F16)}
  m = OracleModel(cfg, w, compress, precision)
  m._tables(Kc.shape[1])
  out = m.decode_layer(m.layers[0], np.asarray(h, F16).astype(F32).reshape(1, -1), Kc, Vc, pos)
  return out.astype(F16)


def random_llama_weights(cfg: Config, seed: int = 0, std: float = 0.02, dtype=F16, moe: bool = False,
                         qkv_bias: bool = False, shared_expert: int = 0):
  """Seeded N(0, std) weights in the reference layout, unit norms (the shape of
  `tests/_helpers.py:make_random_llama_model`, with the benchmark's N(0, 0.02)). `shared_expert` > 0
  adds a Qwen2-MoE shared expert of that width and its sigmoid gate to every MoE layer (the keys
  `aneforge/moe.py:165-167` loads)."""
  rng = np.random.default_rng(seed)
  R = lambda *s: (rng.standard_normal(s, dtype=F32) * F32(std)).astype(dtype)
  dh, D = cfg.dh, cfg.dim
  w = {"embed": R(cfg.vocab, D), "final_norm": np.ones(D, F32), "lm_head": R(cfg.vocab, D), "layers": []}
  for _ in range(cfg.n_layers):
    lw = {"wq": R(cfg.n_heads * dh, D), "wk": R(cfg.n_kv_heads * dh, D), "wv": R(cfg.n_kv_heads * dh, D),
          "wo": R(D, cfg.n_heads * dh), "attn_norm": np.ones(D, F32), "mlp_norm": np.ones(D, F32)}
    if qkv_bias:
      lw["q_bias"] = R(cfg.n_heads * dh); lw["k_bias"] = R(cfg.n_kv_heads * dh); lw["v_bias"] = R(cfg.n_kv_heads * dh)
    if moe:
      E = cfg.extra["n_experts"]
      lw["router"] = R(E, D)
      lw["wgate_exps"] = R(E, cfg.ffn_dim, D); lw["wup_exps"] = R(E, cfg.ffn_dim, D)
      lw["wdown_exps"] = R(E, cfg.ffn_dim, D)
      if shared_expert:
        Fs = int(shared_expert)
        lw["wgate_sh"] = R(Fs, D); lw["wup_sh"] = R(Fs, D); lw["wdown_sh"] = R(D, Fs); lw["shared_gate"] = R(1, D)
    else:
      lw["wgate"] = R(cfg.ffn_dim, D); lw["wup"] = R(cfg.ffn_dim, D); lw["wdown"] = R(D, cfg.ffn_dim)
    w["layers"].append(lw)
  return w
