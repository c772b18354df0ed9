"""Greedy speculative decoding on the device (the reference's `aneforge/speculative.py:131-165`,
`spec_generate`): a small draft model proposes `n_draft` tokens, the target checks all of them in
ONE multi-token verify step over its resident cache, and the matching prefix plus one corrected (or
bonus) token are emitted. Greedy speculative decoding is exact: it emits the target's greedy tokens.

B200 form:
  * the draft's proposals are `n_draft` back-to-back replays of its decode program with the token
    fed back on the device (no host round trip between them), read once from its token history;
  * the target's verify is the decode step over Kq = n_draft + 1 rows that are consecutive tokens of
    one sequence sharing one cache (`LlamaPrefill._verifier`): each row appends its K / V first and
    attends up to its own position, the head's greedy argmax gives the target's token after each;
  * both caches are seeded by their batched prefill; rejected draft positions are overwritten in the
    next round (the reference's incremental scheme), the target's too (the next verify rewrites from
    the first unconfirmed position on before any row reads it).
"""
from __future__ import annotations

import numpy as np

import torch

from .llm import LlamaPrefill


def _argmax_rows(target: LlamaPrefill, ver) -> list:
  """The target's greedy token after each verify row: the device argmax when the head is exactly fp16
  (it then equals the host fp32 head's argmax), else the host logits with the reference's tie-margin
  recheck on each row."""
  prog = ver["prog"]
  if target._head_exact:
    return [int(t) for t in prog.read_output("tok_out")]
  hid = prog.read_output("hid")
  return [int(np.argmax(target._decode_logits(h, None, True))) for h in hid]


def spec_generate(target: LlamaPrefill, draft: LlamaPrefill, token_ids, max_new_tokens=40, eos_id=None,
                  max_len=None, n_draft=4, on_token=None, stats: dict | None = None):
  """Greedy speculative decoding (reference signature): the same tokens as `target.generate(...)`,
  with the target run once per accepted run of draft tokens. `stats`, when given, receives the
  number of verify steps and of accepted draft tokens."""
  prompt = [int(t) for t in token_ids]
  target._check_ids(prompt)
  P = len(prompt)
  M = int(max_len or P + max_new_tokens)
  Kq = int(n_draft) + 1
  eos = {int(eos_id)} if isinstance(eos_id, int) else {int(e) for e in (eos_id or ())}
  ver = target._verifier(M, Kq)
  dec = draft._decoder(M, 1)
  vprog, dprog = ver["prog"], dec["prog"]
  with torch.cuda.device(target.device):
    torch.cuda.synchronize()
    target._reset_state(ver)
  with torch.cuda.device(draft.device):
    draft._reset_state(dec)
  # both caches from their batched prefills; the first token is the target's greedy choice
  pre, real, _ = target._prefill_hidden(prompt)
  hid = pre["prog"].read_output("hid")
  cur = int(np.argmax(target._decode_logits(hid[real - 1], None, True)))
  with torch.cuda.device(target.device):
    target._seed_cache(ver, pre, real)
    torch.cuda.synchronize()
  dpre, dreal, _ = draft._prefill_hidden(prompt)
  with torch.cuda.device(draft.device):
    draft._seed_cache(dec, dpre, dreal)
    torch.cuda.synchronize()
  out = [cur]
  n_verify = n_accept = 0
  if cur in eos:
    return out
  if on_token is not None:
    on_token(cur)
  p = P                                                       # position of `cur`
  while len(out) < max_new_tokens and p + Kq < M:
    # the draft proposes n_draft tokens from cur (device-resident feedback)
    dprog.set_input("tok", np.array([cur], np.int32))
    dprog.set_input("pos", np.array([p], np.int32))
    for _ in range(n_draft):
      dprog.execute_async()
    dprog.sync()
    drafts = [int(t) for t in dprog.read_output("hist")[0][p:p + n_draft]]
    # one verify step over cur + drafts at positions p .. p + n_draft
    vprog.set_input("tok", np.array([cur] + drafts, np.int32))
    vprog.set_input("pos", np.arange(p, p + Kq, dtype=np.int32))
    vprog.execute()
    n_verify += 1
    g = _argmax_rows(target, ver)
    a = 0
    while a < n_draft and g[a] == drafts[a]:
      a += 1
    n_accept += a
    if a == n_draft:
      # every draft accepted: give the draft's cache the last proposal too (row p + n_draft)
      dprog.set_input("tok", np.array([drafts[-1]], np.int32))
      dprog.set_input("pos", np.array([p + n_draft], np.int32))
      dprog.execute()
    emit = drafts[:a] + [g[a]]
    for t in emit:
      if len(out) >= max_new_tokens:
        break
      out.append(t)
      if t in eos:
        break
      if on_token is not None:
        on_token(t)
    if out[-1] in eos:
      break
    cur, p = emit[-1], p + a + 1
  if stats is not None:
    stats.update(verify_steps=n_verify, accepted=n_accept)
  return out[:max_new_tokens]
