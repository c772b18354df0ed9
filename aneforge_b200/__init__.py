"""aneforge_b200: a B200-native (sm_100a) drop-in for ANEForge's quantized LLM inference hot path.

`compile(graph, compress=...)` / `compile_multi`, `load_llm` / `llm.LlamaPrefill.generate` and the
compress= weight policy keep the reference's surface; the work runs as hand-written CUDA kernels
sequenced by the C-ABI program runtime in `_lib/libaf_cuda.so`. There is no CPU fallback: without a
CUDA device the runtime raises.
"""
from . import graph  # noqa: F401
from . import llm  # noqa: F401
from . import moe  # noqa: F401  (registers the "moe" MLP with the runner)
from . import hybrid  # noqa: F401  (registers the gated DeltaNet / gated attention mixers)
from ._compile import Model, MultiModel, compile, compile_multi  # noqa: F401,A004
from .graph import Tensor, concat, const, gather, input, maximum, minimum, select, split, stack, where  # noqa: F401,A004
from .llm import LlamaConfig, LayerSpec, LlamaPrefill, from_pretrained, rope_tables  # noqa: F401

load_llm = from_pretrained

__all__ = ["llm", "graph", "compile", "compile_multi", "Model", "MultiModel", "Tensor", "input", "const", "concat",
           "select", "where", "maximum", "minimum", "split", "stack", "gather", "LlamaConfig", "LayerSpec",
           "LlamaPrefill", "load_llm", "from_pretrained", "rope_tables"]
