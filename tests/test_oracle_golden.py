"""Pin the CPU oracle to the reference: every golden vector the reference produced
(tests/golden/make_golden.py) must be reproduced by the numpy restatement in `oracle/`.

Quantizer bytes are compared bit-exactly; decode/prefill logits in the oracle's fp32 mode are
compared tightly (same math, different summation order), greedy tokens exactly.
"""
import numpy as np
import pytest

from oracle import quant as Q
from oracle.model import OracleModel, rms_consts, topk_gate, Config
from tests._golden import load, llm_case

F16, F32 = np.float16, np.float32


@pytest.fixture(scope="module")
def qz():
  return load("quant.npz")


def test_quantize_per_row_bytes(qz):
  for W, key in ((qz["W"], "per_row"), (qz["W16"], "per_row16")):
    q, s = Q.quantize_per_row(W)
    assert np.array_equal(q.reshape(-1), qz[f"{key}_q"])
    assert np.array_equal(s.view(np.uint16), qz[f"{key}_s"].view(np.uint16))


def test_quantize_per_row_zero_row_and_ties(qz):
  q, s = Q.quantize_per_row(qz["W"])
  assert np.all(q[3] == 0) and np.float32(s[3]) == np.float32(np.float16(1e-8))
  assert q[5].max() == 127 and q[5].min() == -127


def test_palettize_lut4_bytes(qz):
  p, lut = Q.palettize_lut4(qz["Wl"])
  assert np.array_equal(p.reshape(-1), qz["lut4_packed"])
  assert np.array_equal(lut.view(np.uint16), qz["lut4_lut"].view(np.uint16))
  p, lut = Q.palettize_lut4(qz["Wo"])                      # odd IN pads each row with index 0
  assert np.array_equal(p.reshape(-1), qz["lut4o_packed"])
  assert np.array_equal(lut.view(np.uint16), qz["lut4o_lut"].view(np.uint16))


def test_quantize_blockwise_bytes(qz):
  q, s, nb = Q.quantize_blockwise(qz["W"], 32)
  assert nb == int(qz["bw_nb"]) and np.array_equal(q.reshape(-1), qz["bw_q"])
  assert np.array_equal(s.reshape(-1).view(np.uint16), qz["bw_s"].view(np.uint16))
  q, s, nb = Q.quantize_blockwise(qz["Wi"], 32)            # indivisible: block clamps to a divisor
  assert nb == int(qz["bwi_nb"]) == 3
  assert np.array_equal(q.reshape(-1), qz["bwi_q"])
  assert np.array_equal(s.reshape(-1).view(np.uint16), qz["bwi_s"].view(np.uint16))


def test_sparsify_bytes(qz):
  m, v = Q.sparsify(qz["Ws"])
  assert np.array_equal(m, qz["sp_mask"]) and np.array_equal(v.view(np.uint16), qz["sp_vals"].view(np.uint16))


@pytest.mark.parametrize("name", ["W", "Ws", "Mx", "Wl"])
@pytest.mark.parametrize("mode", ["None", "int8", "int4", "blockwise", "sparse", "auto"])
def test_encoding_decision_matches_reference(qz, name, mode):
  M = qz["W16"] if False else {"W": qz["W"], "Ws": qz["Ws"], "Wl": qz["Wl"],
                               "Mx": np.repeat(np.eye(4, dtype=F16), 2, axis=0)}[name]
  enc = Q.encode_weight(M, None if mode == "None" else mode)
  assert enc.kind == str(qz[f"enc_{name}_{mode}_kind"])
  np.testing.assert_array_equal(enc.deq.astype(F32), qz[f"enc_{name}_{mode}_deq"])


@pytest.mark.parametrize("D,eps", [(64, 1e-5), (4096, 1e-5), (128, 1e-6)])
def test_rms_constants(qz, D, eps):
  g, floor = rms_consts(qz[f"rms_{D}_{eps}_gamma"], eps)
  assert np.array_equal(g.view(np.uint16), qz[f"rms_{D}_{eps}_g"].view(np.uint16))
  assert np.float16(floor).view(np.uint16) == qz[f"rms_{D}_{eps}_floor"].view(np.uint16)


def test_g32_int4_roundtrip():
  """Group-32 int4 has no reference counterpart (parity unpinned): check its own contract."""
  rng = np.random.default_rng(0)
  W = (rng.standard_normal((16, 128)) * 0.02).astype(F32)
  p, s = Q.quantize_g32_int4(W)
  assert p.shape == (16, 64) and s.shape == (16, 4)
  nib = np.stack([p & 15, p >> 4], -1).reshape(16, 128)
  assert nib.min() >= 1 and nib.max() <= 15
  R = Q.dequant_g32_int4(p, s)
  rel = np.linalg.norm(R - W) / np.linalg.norm(W)
  assert rel < 0.12


@pytest.mark.parametrize("tag", ["int8", "int8_tbt", "fp16", "int4", "bias_qknorm", "mha"])
def test_oracle_generate_matches_reference(tag):
  cfg, w, z = llm_case(tag)
  comp = str(z["compress"]); comp = None if comp == "None" else comp
  m = OracleModel(cfg, w, comp, precision="fp32")
  toks, lg = m.generate(list(z["prompt"]), int(z["n_new"]), max_len=int(z["max_len"]) or None,
                        batched_prefill=bool(z["batched"]), prefill_pad=int(z["pad"]) or None,
                        return_logits=True)
  assert toks == list(z["tokens"])
  ref = z["logits"]
  got = np.stack(lg)
  assert got.shape == ref.shape
  err = np.abs(got - ref).max() / np.abs(ref).max()
  assert err < 2e-3, err                                   # fp16 port roundings differ by 1 ulp at most
  # device-precision mode stays within the fp16 tolerance of the reference
  md = OracleModel(cfg, w, comp, precision="device")
  _, lgd = md.generate(list(z["prompt"]), int(z["n_new"]), max_len=int(z["max_len"]) or None,
                       batched_prefill=bool(z["batched"]), prefill_pad=int(z["pad"]) or None,
                       return_logits=True)
  d = np.stack(lgd)
  cos = float((d.ravel() @ ref.ravel()) / (np.linalg.norm(d) * np.linalg.norm(ref)))
  assert cos > 0.999


def test_oracle_prefill_matches_reference():
  cfg, w, z = llm_case("int8")
  m = OracleModel(cfg, w, "int8", precision="fp32")
  hid, _ = m.prefill_hidden(list(z["prompt"]))
  lg = m.logits(hid[-1].astype(F32))
  ref = z["prefill_logits"].reshape(-1)
  assert np.abs(lg - ref).max() / np.abs(ref).max() < 2e-3


def test_topk_gate_exact_ties():
  z = load("moe.npz")
  got = topk_gate(z["topk_rows"].astype(F32), 2)
  np.testing.assert_array_equal(got.astype(F16), z["topk_out"].astype(F16))


@pytest.mark.parametrize("compress", ["None", "int8"])
@pytest.mark.parametrize("T", [1, 5])
def test_moe_layer_matches_reference(compress, T):
  z = load("moe.npz")
  lw = {k: z[k] for k in ("mlp_norm", "router", "wgate_exps", "wup_exps", "wdown_exps")}
  cfg = Config(dim=64, n_layers=1, n_heads=4, n_kv_heads=2, ffn_dim=32, vocab=16,
               extra={"n_experts": 8, "n_experts_per_tok": 2, "norm_topk_prob": True})
  lw.update(wq=np.zeros((64, 64), F16), wk=np.zeros((32, 64), F16), wv=np.zeros((32, 64), F16),
            wo=np.zeros((64, 64), F16), attn_norm=np.ones(64, F32))
  w = {"embed": np.zeros((16, 64), F16), "final_norm": np.ones(64, F32), "lm_head": np.zeros((16, 64), F16),
       "layers": [lw]}
  m = OracleModel(cfg, w, None if compress == "None" else compress, precision="fp32")
  h = z[f"h_{compress}_{T}"].astype(F32)
  y = m._mlp(m.layers[0], h).astype(F16).astype(F32)
  ref = z[f"y_{compress}_{T}"]
  assert np.abs(y - ref).max() / np.abs(ref).max() < 2e-3
