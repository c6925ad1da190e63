"""mlx_qsdpa on B200: fused quantized-KV decode attention on PyTorch CUDA tensors.

Drop-in for the public API of Thump604/mlx-qsdpa (mlx_qsdpa/__init__.py:1-78):
``quantized_sdpa``, ``cache_sdpa`` and the four quantized cache classes, with
torch tensors in place of ``mx.array``.  The kernels are hand-written sm_100a
CUDA in ``libqsdpa.so`` (C ABI: include/qsdpa.h), loaded through ctypes by
``mlx_qsdpa._lib``.
"""

from .dispatch import DEFAULT_THRESHOLD, KVRanges, dequant_sdpa, quantized_sdpa
from .cache import (
    QuantizedSDPACache,
    BatchQuantizedSDPACache,
    QuantizedRotatingSDPACache,
    BatchQuantizedRotatingSDPACache,
)
from .serialize import load_prompt_cache, save_prompt_cache

__version__ = "0.3.1+b200"

# Sequence length at which cache_sdpa switches from dequantise + SDPA to the
# fused kernel.  The reference's 16384 was measured on an M2 Ultra
# (__init__.py:19, README.md "Dynamic dispatch crossover"); on B200 the fused
# kernel wins from the shortest contexts, so decode always takes it.
DEFAULT_CROSSOVER = 0


def cache_sdpa(
    q,
    k_quant,
    v_quant,
    cache,
    scale=None,
    mask=None,
    crossover=DEFAULT_CROSSOVER,
):
    """Attention with dynamic dispatch: dequant + SDPA below ``crossover``, fused above.

    Restates mlx_qsdpa/__init__.py:12-68: prefill (qL > 1) or N < crossover
    dequantises K/V with the cache's bits/group_size and runs SDPA; otherwise
    the fused kernel runs with the cache's quantisation parameters.

    Args:
        q:         (B, H_q, qL, D) float16/bfloat16 query
        k_quant:   (packed_uint32, scales, biases) from the cache
        v_quant:   (packed_uint32, scales, biases) from the cache
        cache:     any of the four quantized caches (provides bits, group_size)
        scale:     attention scale (default 1/sqrt(D))
        mask:      None, "causal", bool/additive tensor, or KVRanges
        crossover: sequence length from which decode uses the fused kernel
    """
    D = q.shape[-1]
    qL = q.shape[2]
    N = k_quant[0].shape[2]
    if scale is None:
        scale = D ** -0.5
    if qL > 1 or N < crossover:
        return dequant_sdpa(q, k_quant[0], v_quant[0], k_quant[1], v_quant[1], k_quant[2], v_quant[2],
                            scale, mask, cache.bits, cache.group_size)
    return quantized_sdpa(
        q, k_quant[0], v_quant[0],
        k_quant[1], v_quant[1], k_quant[2], v_quant[2],
        scale=scale, mask=mask,
        bits=cache.bits, group_size=cache.group_size,
    )


__all__ = [
    "quantized_sdpa",
    "QuantizedSDPACache",
    "BatchQuantizedSDPACache",
    "QuantizedRotatingSDPACache",
    "BatchQuantizedRotatingSDPACache",
    "cache_sdpa",
    "KVRanges",
    "save_prompt_cache",
    "load_prompt_cache",
]
