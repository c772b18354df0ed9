"""CPU oracle for the quantized LLM decode/prefill hot path.

TEST INFRASTRUCTURE ONLY. This package is a plain-numpy restatement of the reference
(sbryngelson/ANEForge) algorithm for the path that `aneforge_b200` runs on the GPU:

  * `oracle.quant`  - the weight encoders of `aneforge/_blob.py` and the encoding decision of
                      `aneforge/_compile.py:_Emitter.weight`, plus the group-32 int4 format.
  * `oracle.model`  - the decoder numerics of `aneforge/llm.py` (RMSNorm lowering, RoPE tables,
                      GQA decode/prefill attention, SwiGLU, lm_head, greedy/sampled generate) and
                      the MoE layer of `aneforge/moe.py`.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s `cpu_baseline` / `--impl reference`
leg may import it, and only as the checker or as the timed CPU baseline. The product package
`aneforge_b200` never imports it.

Parity pins: the restatement is checked against golden vectors produced by the reference's own
code (`tests/golden/make_golden.py`, run in a container that has the reference mounted) by
`tests/test_oracle_golden.py`. The group-32 int4 format has no reference implementation and is
"parity unpinned".
"""
