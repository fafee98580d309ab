"""Host-side argument checks of the PyTorch wrapper (no GPU: meta and CPU tensors).

Every output, value and temp tensor is checked against the keys before any CUDA call, since the
kernels write exactly the input's bytes into the outputs."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from libcusort_b200.torch_sort import _check_args, radix_sort  # noqa: E402

M = "meta"


def _k(n=10, dtype=torch.int32):
    return torch.empty(n, dtype=dtype, device=M)


def test_cpu_tensor_is_rejected():
    with pytest.raises(ValueError, match="CUDA"):
        radix_sort(torch.arange(10, dtype=torch.int32))


def test_value_widths():
    k = _k(10)
    assert _check_args(k, None, None, None, None) == 0
    assert _check_args(k, torch.empty(10, dtype=torch.int8, device=M), None, None, None) == 1
    assert _check_args(k, torch.empty(10, 2, dtype=torch.int64, device=M), None, None, None) == 16
    assert _check_args(k, torch.empty(10, 2, dtype=torch.int16, device=M), None, None, None) == 4
    with pytest.raises(ValueError, match="3 bytes"):
        _check_args(k, torch.empty(10, 3, dtype=torch.uint8, device=M), None, None, None)
    with pytest.raises(ValueError, match="leading dimension"):
        _check_args(k, torch.empty(11, dtype=torch.int32, device=M), None, None, None)


def test_empty_inputs_keep_their_value_width():
    k = _k(0)
    assert _check_args(k, torch.empty(0, 2, dtype=torch.int64, device=M), None, None, None) == 16
    assert _check_args(k, torch.empty(0, dtype=torch.int32, device=M), None, None, None) == 4


def test_outputs_must_match_inputs():
    k = _k(10)
    v = torch.empty(10, dtype=torch.int64, device=M)
    with pytest.raises(ValueError, match="out_keys"):
        _check_args(k, None, _k(9), None, None)
    with pytest.raises(ValueError, match="out_keys"):
        _check_args(k, None, _k(10, torch.float32), None, None)
    with pytest.raises(ValueError, match="out_keys"):
        _check_args(k, None, torch.empty(20, dtype=torch.int32, device=M)[::2], None, None)
    with pytest.raises(ValueError, match="out_values"):
        _check_args(k, v, None, torch.empty(10, dtype=torch.int32, device=M), None)
    with pytest.raises(ValueError, match="out_values given without values"):
        _check_args(k, None, None, v, None)
    assert _check_args(k, v, _k(10), torch.empty_like(v), None) == 8


def test_devices_and_temp():
    k = _k(10)
    with pytest.raises(ValueError, match="values are on"):
        _check_args(k, torch.empty(10, dtype=torch.int32), None, None, None)
    with pytest.raises(ValueError, match="out_keys"):
        _check_args(k, None, torch.empty(10, dtype=torch.int32), None, None)
    with pytest.raises(ValueError, match="temp"):
        _check_args(k, None, None, None, torch.empty(100, dtype=torch.int32, device=M))
    with pytest.raises(ValueError, match="temp"):
        _check_args(k, None, None, None, torch.empty(100, dtype=torch.uint8))
    assert _check_args(k, None, None, None, torch.empty(100, dtype=torch.uint8, device=M)) == 0


def test_key_shape_and_dtype():
    with pytest.raises(ValueError, match="1-D"):
        _check_args(torch.empty(2, 5, dtype=torch.int32, device=M), None, None, None, None)
    with pytest.raises(TypeError, match="unsupported key dtype"):
        _check_args(torch.empty(5, dtype=torch.bool, device=M), None, None, None, None)


def test_sharded_output_capacity():
    from libcusort_b200.mgpu import _check_output
    k = _k(10)
    _check_output("out_keys", _k(64), k, 64)
    with pytest.raises(ValueError, match="capacity=64"):
        _check_output("out_keys", _k(63), k, 64)
    with pytest.raises(ValueError, match="out_keys"):
        _check_output("out_keys", _k(64, torch.int64), k, 64)
    v = torch.empty(10, 2, dtype=torch.int64, device=M)
    _check_output("out_values", torch.empty(64, 2, dtype=torch.int64, device=M), v, 64)
    with pytest.raises(ValueError, match="out_values"):
        _check_output("out_values", torch.empty(128, dtype=torch.int64, device=M), v, 64)


def test_segment_offsets_checks():
    from libcusort_b200.torch_sort import _check_offsets
    k = _k(10)
    b = torch.empty(4, dtype=torch.int64, device=M)
    assert _check_offsets(k, b, b) == 4
    with pytest.raises(ValueError, match="begin_offsets"):
        _check_offsets(k, torch.empty(4, dtype=torch.int32, device=M), b)
    with pytest.raises(ValueError, match="end_offsets"):
        _check_offsets(k, b, torch.empty(4, dtype=torch.int64))
    with pytest.raises(ValueError, match="same length"):
        _check_offsets(k, b, torch.empty(5, dtype=torch.int64, device=M))


def test_any_width_payloads_only_where_allowed():
    k = _k(10)
    v = torch.empty(10, 3, dtype=torch.int64, device=M)  # 24 bytes per row
    assert _check_args(k, v, None, None, None, any_width=True) == 24
    with pytest.raises(ValueError, match="24 bytes"):
        _check_args(k, v, None, None, None)


def test_host_sort_rejects_cuda_and_bad_widths():
    from libcusort_b200.torch_sort import radix_sort_host
    with pytest.raises(ValueError, match="CPU"):
        radix_sort_host(_k(10), torch.empty(10, dtype=torch.int32, device=M))
    with pytest.raises(ValueError):
        radix_sort_host(torch.arange(10, dtype=torch.int32), torch.empty(10, 3, dtype=torch.int8))
