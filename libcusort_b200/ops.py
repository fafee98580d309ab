"""PyTorch operators over the C ABI: ``torch.ops.cusort.*``.

Importing this module registers, in the ``cusort`` namespace:

* ``sort_keys(Tensor keys, bool descending=False, int begin_bit=0, int end_bit=-1) -> Tensor``
* ``sort_pairs(Tensor keys, Tensor values, bool descending=False, int begin_bit=0, int end_bit=-1)
  -> (Tensor, Tensor)``
* ``argsort(Tensor keys, bool descending=False) -> Tensor`` (int64 indices)
* ``segmented_sort_keys(Tensor keys, Tensor begin_offsets, Tensor end_offsets, bool descending=False,
  int begin_bit=0, int end_bit=-1) -> Tensor``
* ``segmented_sort_pairs(Tensor keys, Tensor values, Tensor begin_offsets, Tensor end_offsets,
  bool descending=False, int begin_bit=0, int end_bit=-1) -> (Tensor, Tensor)``

``sort_pairs`` takes payload rows of any width (rows of 1, 2, 4, 8 or 16 bytes move with the keys,
others are gathered by the sorted permutation).  The segmented operators sort every segment
[begin_offsets[s], end_offsets[s]) (int64 offsets, non-overlapping) independently; positions
outside every segment keep their input.

All of them are stable, allocate fresh outputs (the inputs are never written), run on torch's current
CUDA stream through ``cusort_sort_keys[_descending]`` / ``cusort_sort_pairs[_descending]`` and have
fake (meta) implementations, so they trace under ``torch.compile`` / ``torch.export`` as opaque
calls.  ``end_bit = -1`` means all key bits.  There is no CPU implementation: a CPU tensor raises.
Floating-point keys follow the radix (IEEE total) order of the reference: -0.0 sorts before +0.0
and NaNs by sign and payload, where ``torch.sort`` treats the zeros as equal.
"""
from __future__ import annotations

import torch

from .torch_sort import radix_sort, segmented_sort


def _end(keys: torch.Tensor, end_bit: int) -> int:
    return 8 * keys.element_size() if end_bit < 0 else end_bit


@torch.library.custom_op("cusort::sort_keys", mutates_args=())
def sort_keys(keys: torch.Tensor, descending: bool = False, begin_bit: int = 0, end_bit: int = -1) -> torch.Tensor:
    k, _ = radix_sort(keys, None, descending=descending, begin_bit=begin_bit, end_bit=_end(keys, end_bit))
    return k


@sort_keys.register_fake
def _(keys, descending=False, begin_bit=0, end_bit=-1):
    return torch.empty_like(keys)


@torch.library.custom_op("cusort::sort_pairs", mutates_args=())
def sort_pairs(keys: torch.Tensor, values: torch.Tensor, descending: bool = False, begin_bit: int = 0,
               end_bit: int = -1) -> tuple[torch.Tensor, torch.Tensor]:
    k, v = radix_sort(keys, values, descending=descending, begin_bit=begin_bit, end_bit=_end(keys, end_bit))
    return k, v


@sort_pairs.register_fake
def _(keys, values, descending=False, begin_bit=0, end_bit=-1):
    return torch.empty_like(keys), torch.empty_like(values)


@torch.library.custom_op("cusort::argsort", mutates_args=())
def argsort(keys: torch.Tensor, descending: bool = False) -> torch.Tensor:
    idx = torch.arange(keys.numel(), device=keys.device, dtype=torch.int64)
    _, perm = radix_sort(keys, idx, descending=descending)
    return perm


@argsort.register_fake
def _(keys, descending=False):
    return torch.empty(keys.shape, dtype=torch.int64, device=keys.device)


@torch.library.custom_op("cusort::segmented_sort_keys", mutates_args=())
def segmented_sort_keys(keys: torch.Tensor, begin_offsets: torch.Tensor, end_offsets: torch.Tensor,
                        descending: bool = False, begin_bit: int = 0, end_bit: int = -1) -> torch.Tensor:
    k, _ = segmented_sort(keys, begin_offsets, end_offsets, None, descending=descending, begin_bit=begin_bit,
                          end_bit=_end(keys, end_bit))
    return k


@segmented_sort_keys.register_fake
def _(keys, begin_offsets, end_offsets, descending=False, begin_bit=0, end_bit=-1):
    return torch.empty_like(keys)


@torch.library.custom_op("cusort::segmented_sort_pairs", mutates_args=())
def segmented_sort_pairs(keys: torch.Tensor, values: torch.Tensor, begin_offsets: torch.Tensor,
                         end_offsets: torch.Tensor, descending: bool = False, begin_bit: int = 0,
                         end_bit: int = -1) -> tuple[torch.Tensor, torch.Tensor]:
    k, v = segmented_sort(keys, begin_offsets, end_offsets, values, descending=descending, begin_bit=begin_bit,
                          end_bit=_end(keys, end_bit))
    return k, v


@segmented_sort_pairs.register_fake
def _(keys, values, begin_offsets, end_offsets, descending=False, begin_bit=0, end_bit=-1):
    return torch.empty_like(keys), torch.empty_like(values)
