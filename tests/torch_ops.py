"""PyTorch custom operators over the C ABI, for the test harness only (the
library's callers use the C ABI, the C++ API or the ctypes wrappers in
gemma4metal_b200.turboquant): torch.ops.tq.quantize_append mutates the cache
in place, torch.ops.tq.sdpa_int4 returns the attention output."""
from typing import Tuple

import torch

import gemma4metal_b200.turboquant as tq


@torch.library.custom_op("tq::quantize_append", mutates_args=("k_quant", "k_scales", "k_biases",
                                                               "v_quant", "v_scales", "v_biases"))
def quantize_append(k_new: torch.Tensor, v_new: torch.Tensor, k_quant: torch.Tensor,
                    k_scales: torch.Tensor, k_biases: torch.Tensor, v_quant: torch.Tensor,
                    v_scales: torch.Tensor, v_biases: torch.Tensor, pos: int) -> None:
    tq.quantize_append(k_new, v_new, k_quant, k_scales, k_biases, v_quant, v_scales, v_biases,
                       pos=pos, s=torch.cuda.current_stream())


@torch.library.custom_op("tq::sdpa_int4", mutates_args=())
def sdpa_int4(queries: torch.Tensor, k_quant: torch.Tensor, k_scales: torch.Tensor,
              k_biases: torch.Tensor, v_quant: torch.Tensor, v_scales: torch.Tensor,
              v_biases: torch.Tensor, gqa_factor: int, scale: float, sliding_window: int,
              n_tokens: int) -> torch.Tensor:
    return tq.sdpa_int4(queries, k_quant, k_scales, k_biases, v_quant, v_scales, v_biases,
                        gqa_factor, scale, sliding_window, torch.cuda.current_stream(),
                        n_tokens=n_tokens)


@sdpa_int4.register_fake
def _sdpa_int4_fake(queries, k_quant, k_scales, k_biases, v_quant, v_scales, v_biases,
                    gqa_factor, scale, sliding_window, n_tokens):
    return torch.empty_like(queries)


def cache_tensors(cache) -> Tuple[torch.Tensor, ...]:
    return tuple(cache.tensors())
