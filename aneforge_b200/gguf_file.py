"""Read access to a GGUF checkpoint for the model loaders (reference `aneforge/_gguf.py:10-48`): the
architecture, its scoped metadata scalars, and tensors by name dequantized to numpy.

Tensors come back in the reader's numpy order, which is the PyTorch [out, in] order (GGUF stores the
dimensions innermost first). Quantized GGUF tensors (Q8_0, Q4_K, ...) are expanded with the `gguf`
package's own dequantizer: the device formats are produced afterwards by the graph's `compress=`,
exactly as the reference re-encodes its fp16 weights."""
from __future__ import annotations

import mmap
from typing import Any

import numpy as np


class GGUFFile:
  def __init__(self, path: str):
    try:
      import gguf
      from gguf.quants import dequantize
    except ImportError as e:                     # the reference needs the same package
      raise ImportError("reading GGUF checkpoints needs the `gguf` package") from e
    self._dequantize = dequantize
    self._plain = (gguf.GGMLQuantizationType.F32, gguf.GGMLQuantizationType.F16)
    self.reader = gguf.GGUFReader(path)
    self.fields = dict(self.reader.fields)
    counts = [k for k in self.fields if k.endswith(".block_count")]
    if not counts:
      raise ValueError(f"{path}: no '<arch>.block_count' metadata")
    self.arch = counts[0].split(".", 1)[0]
    self.tensors = {t.name: t for t in self.reader.tensors}

  def field(self, key: str, default: Any = None) -> Any:
    """A scalar metadata value by its full key, or `default`."""
    f = self.fields.get(key)
    if f is None:
      return default
    v = f.contents()
    return v.item() if isinstance(v, np.generic) else v

  def scalar(self, key: str, default: Any = None) -> Any:
    """A scalar of this architecture (`scalar("block_count")` reads `<arch>.block_count`)."""
    return self.field(f"{self.arch}.{key}", default)

  def has(self, name: str) -> bool:
    return name in self.tensors

  def shape(self, name: str) -> tuple:
    """GGUF dimension order, innermost first (e.g. [dim, ffn, E] for an expert gate tensor)."""
    return tuple(int(x) for x in self.tensors[name].shape)

  def rows(self, name: str) -> int:
    return int(np.asarray(self.tensors[name].data).shape[0])

  def get(self, name: str, dtype=np.float16) -> np.ndarray:
    t = self.tensors[name]
    d = np.asarray(t.data)
    if t.tensor_type not in self._plain:
      d = self._dequantize(d, t.tensor_type)
    return np.ascontiguousarray(d.astype(dtype, copy=False))

  def release_pages(self) -> None:
    """Drop the file's mapped pages once a layer has been copied out, so the raw checkpoint and its
    dequantized layers are not both resident."""
    mm = getattr(self.reader.data, "_mmap", None)
    if mm is not None:
      try:
        mm.madvise(mmap.MADV_DONTNEED)
      except (AttributeError, OSError, ValueError):
        pass


class LazyLayers:
  """Per-layer host weights made on first use and dropped by `free(i)` once the runner has encoded
  them onto the device, so a checkpoint larger than host RAM loads one layer at a time."""

  def __init__(self, make, n: int):
    self._make, self._n, self._have = make, int(n), {}

  def __len__(self) -> int:
    return self._n

  def __getitem__(self, i: int) -> dict:
    if not -self._n <= i < self._n:
      raise IndexError(i)
    i %= self._n
    if i not in self._have:
      self._have[i] = self._make(i)
    return self._have[i]

  def __iter__(self):
    return (self[i] for i in range(self._n))

  def free(self, i: int) -> None:
    self._have.pop(i, None)
