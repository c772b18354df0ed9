"""Plan builder: emits the text plan libaf_cuda.so compiles into a program (see csrc/program.cu for
the grammar). A plan is the B200 counterpart of the reference's MIL program text
(`aneforge/_compile.py:906-923`): named ports, weights and one fused kernel launch per line."""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class Buf:
  name: str
  nbytes: int
  role: str               # in | out | state | tmp | weight | scratch


@dataclass
class PlanBuilder:
  bufs: dict = field(default_factory=dict)
  ops: list = field(default_factory=list)
  wfile: dict = field(default_factory=dict)

  def buf(self, name: str, nbytes: int, role: str) -> str:
    if role not in ("in", "out", "state", "tmp", "weight", "scratch"):
      raise ValueError(role)
    nbytes = int(nbytes)
    if name in self.bufs:
      b = self.bufs[name]
      if b.role != role:
        raise ValueError(f"buffer {name} redeclared with role {role} (was {b.role})")
      b.nbytes = max(b.nbytes, nbytes)
    else:
      self.bufs[name] = Buf(name, max(nbytes, 1), role)
    return name

  def op(self, kind: str, **kv) -> None:
    for k, v in kv.items():
      if v is None:
        kv[k] = "-"
    self.ops.append((kind, kv))

  def text(self) -> str:
    lines = ["AFPLAN 1"]
    for b in self.bufs.values():
      lines.append(f"buf {b.name} {b.nbytes} {b.role}")
    for name, off in self.wfile.items():
      lines.append(f"wfile {name} {off}")
    for kind, kv in self.ops:
      args = " ".join(f"{k}={_fmt(v)}" for k, v in kv.items())
      lines.append(f"op {kind} {args}")
    return "\n".join(lines) + "\n"


def _fmt(v) -> str:
  if isinstance(v, bool):
    return "1" if v else "0"
  if isinstance(v, float):
    return repr(float(v))
  return str(v)


def at(name: str, offset: int) -> str:
  """A buffer reference with a byte offset."""
  return f"{name}@{int(offset)}" if offset else name
