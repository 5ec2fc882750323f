"""dspark-b200: mlx-dspark's speculative-decoding verify path, rebuilt for NVIDIA B200.

Modules mirror the reference operator surface (``src/mlx_dspark/``):

* :mod:`.skinny_qmm` / :mod:`.small_m_qmm` — small-M affine-quantized matmul and its scoped
  dispatch (K1); :mod:`.wide_gemm` — the wide-M (prefill / batch) quantized GEMM on tcgen05,
* :mod:`.multirow_attn` — multi-row causal GQA verify attention (K2),
* :mod:`.kvcache` / :mod:`.batch_engine` — per-row KV cache with in-place rollback (K3) and
  the ragged continuous-batching step built on the device (K4),
* :mod:`.target` — a Qwen3-shaped dense target whose verify forward chains the fused kernels,
* :mod:`.quant` — MLX-layout affine quantization of device tensors.

All compute runs in ``libdspark.so`` (hand-written sm_100a CUDA) through a C ABI; torch only
holds buffers and streams. Importing the package loads the library and fails loudly when it
is missing.
"""

from . import _lib  # noqa: F401  (loads libdspark.so; raises if absent)
from ._lib import DSparkError, DSparkUnsupported  # noqa: F401

__version__ = "0.1.0"
