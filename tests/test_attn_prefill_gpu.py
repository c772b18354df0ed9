"""The prefill causal attention (`attn_prefill` plan op: rope + cache write, then the tcgen05
flash-attention kernel for head dim 128) against a torch fp32 restatement of the attention over the
very q / K / V the op staged (reference `aneforge/llm.py:149-169`, `_attn_prefill_kv`: softmax of
q k^T / sqrt(dh) under the causal mask, times v; under int8 the GQA expansion factor multiplies K and
V as f16(c * f16(x)), `llm.py:205-211`). The kernel rounds P to fp16 for the MMA; the bound below
allows for that rounding."""
import numpy as np
import pytest
import torch

from aneforge_b200 import _blob
from aneforge_b200 import _runtime as R
from aneforge_b200 import llm
from aneforge_b200.plan import PlanBuilder

pytestmark = pytest.mark.gpu
F16 = np.float16


def _run(S, H, KV, expand, seed):
  dh = 128
  Q = (H + 2 * KV) * dh
  c = _blob.gqa_expand_factor(KV, H // KV, "int8") if expand else 1.0
  pb = PlanBuilder()
  pb.buf("qkv", 4 * S * Q, "in")
  pb.buf("K", 2 * KV * S * dh, "state"); pb.buf("V", 2 * KV * S * dh, "state")
  pb.buf("qbuf", 2 * H * S * dh, "state"); pb.buf("att", 2 * S * H * dh, "out")
  pb.buf("cos", 2 * S * dh, "weight"); pb.buf("sin", 2 * S * dh, "weight")
  kv = dict(qkv="qkv", kc="K", vc="V", out="att", qbuf="qbuf", cos="cos", sin="sin", s=S, h=H, kv=KV, dh=dh, ldm=S,
            scale=float(dh ** -0.5), kvc=c, expand=int(expand))
  if expand:
    kv["kvx"] = pb.buf("kvx", 2 * 2 * KV * S * dh, "state")
  pb.op("attn_prefill", **kv)
  prog = R.Program.from_text(pb.text(), {"qkv": (S, Q)}, {"att": (S, H * dh)}, 0, {"qkv": "fp32"})
  cos_t, sin_t = llm.rope_tables(S, dh, 500000.0)
  prog.upload("cos", np.ascontiguousarray(cos_t, F16)); prog.upload("sin", np.ascontiguousarray(sin_t, F16))
  rng = np.random.default_rng(seed)
  qkv = rng.standard_normal((S, Q)).astype(np.float32)
  qkv[:, :H * dh] *= 2.0                                    # sharper softmax rows
  prog.set_input("qkv", qkv)
  prog.execute()
  out = prog.read_output("att").astype(np.float32).reshape(S, H, dh)
  q = prog.tensor("qbuf", (H, S, dh)).float()
  k = prog.tensor("K", (KV, S, dh)).float()
  v = prog.tensor("V", (KV, S, dh)).float()
  if expand:
    k = (c * k).half().float()
    v = (c * v).half().float()
    kx = prog.tensor("kvx", (2, KV, S, dh)).float()
    assert torch.equal(kx[0], k) and torch.equal(kx[1], v)   # the staged copies are exactly f16(c * f16(x))
  g = H // KV
  k, v = k.repeat_interleave(g, 0), v.repeat_interleave(g, 0)
  sc = torch.einsum("hsd,htd->hst", q, k) * dh ** -0.5
  mask = torch.ones(S, S, dtype=torch.bool, device=sc.device).tril()
  p = torch.softmax(sc.masked_fill(~mask, float("-inf")), dim=-1)
  ref = torch.einsum("hst,htd->shd", p, v).cpu().numpy()
  prog.release()
  return out, ref


@pytest.mark.parametrize("S", [1, 5, 127, 128, 129, 300, 512])
@pytest.mark.parametrize("heads", [(8, 2), (4, 4)])
@pytest.mark.parametrize("expand", [False, True])
def test_prefill_attention_matches_torch(S, heads, expand):
  H, KV = heads
  if expand and H == KV:
    pytest.skip("the expansion factor applies to grouped heads only")
  out, ref = _run(S, H, KV, expand, seed=S + 7 * H)
  err = np.abs(out - ref).max()
  assert err <= 4e-3 * max(1.0, np.abs(ref).max()), err
  cos = (out.ravel() @ ref.ravel()) / (np.linalg.norm(out) * np.linalg.norm(ref))
  assert cos > 0.99999, cos


def test_prefill_attention_replays_identically():
  """Two executions of the same program give the same bytes (no state leaks between CTAs or runs)."""
  a, _ = _run(300, 8, 2, True, seed=3)
  b, _ = _run(300, 8, 2, True, seed=3)
  assert np.array_equal(a, b)
