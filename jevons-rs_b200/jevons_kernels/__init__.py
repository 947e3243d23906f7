"""B200-native GGML quantized matmul (Q8_0 / Q4_K / Q6_K / Q5_0 / F16 weights) for jevons-rs.

Python mirror of the reference's matmul path API over the C ABI in include/jk.h:

  * `formats`  -- jevons-formats: TensorType, block(), q4k_scale_min, packed_words, Packed, pack
  * `gemm`     -- jevons-kernels: Gpu, Buf, QMatrix, Plan, SplitScratch, matmul, matmul_plan,
                  matvec, matmul_tiled; jevons-burn: f16_linear, f16_linear_scaled
  * `synth`    -- seeded synthetic GGML weights and activations with the benchmark shapes
  * `shard`    -- column sharding of a projection across ranks and the all-gather of its outputs
"""
from ._lib import JkError, Plan, load  # noqa: F401
from .formats import Packed, TensorType, block, pack, packed_words, q4k_scale_min  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # gemm imports torch; keep `import jevons_kernels` cheap for format-only users.
    if name in ("gemm",):
        import importlib
        return importlib.import_module(".gemm", __name__)
    raise AttributeError(name)
