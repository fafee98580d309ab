"""torch.ops.cusort.* (libcusort_b200/ops.py): registration and fake shapes on
CPU; on the GPU, equality with torch's own stable sort and tracing under
torch.compile (the operator stays an opaque call)."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

import libcusort_b200.ops  # noqa: E402,F401  (registers the operators)


def test_ops_registered_with_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        k = torch.empty(1000, dtype=torch.float32, device="cuda")
        v = torch.empty(1000, 3, dtype=torch.int32, device="cuda")
        sk, sv = torch.ops.cusort.sort_pairs(k, v, True)
        assert sk.shape == k.shape and sk.dtype == k.dtype
        assert sv.shape == v.shape and sv.dtype == v.dtype
        assert torch.ops.cusort.sort_keys(k).shape == k.shape
        p = torch.ops.cusort.argsort(k)
        assert p.shape == k.shape and p.dtype == torch.int64


def test_cpu_tensor_is_rejected():
    with pytest.raises(ValueError):
        torch.ops.cusort.sort_keys(torch.arange(10, dtype=torch.int32))


gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="no CUDA device")


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.int64, torch.int16, torch.float64])
@pytest.mark.parametrize("descending", [False, True])
def test_ops_match_torch_stable_sort(dtype, descending):
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    if dtype.is_floating_point:
        # many ties; no zeros (the radix order puts -0.0 before +0.0, torch.sort treats them as equal)
        x = torch.randn(200_003, device="cuda", dtype=dtype, generator=g).round(decimals=1) + 0.05
    else:
        x = torch.randint(-50, 50, (200_003,), device="cuda", dtype=dtype, generator=g)
    ref = torch.sort(x, descending=descending, stable=True)
    assert torch.equal(torch.ops.cusort.sort_keys(x, descending), ref.values)
    assert torch.equal(torch.ops.cusort.argsort(x, descending), ref.indices)
    vals = torch.arange(x.numel(), device="cuda", dtype=torch.int32)
    sk, sv = torch.ops.cusort.sort_pairs(x, vals, descending)
    assert torch.equal(sk, ref.values) and torch.equal(sv.long(), ref.indices)


@pytest.mark.gpu
@gpu
def test_ops_under_torch_compile():
    def f(x):
        return torch.ops.cusort.sort_keys(x * 2) + 1

    x = torch.randn(65_537, device="cuda")
    cf = torch.compile(f, backend="aot_eager", fullgraph=True)
    assert torch.equal(cf(x), f(x))


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("n", [0, 1, 2])
def test_ops_tiny_and_empty(n):
    # trivial sizes with a 16-byte payload per item (the payload width comes from the shape,
    # not from numel / n)
    x = torch.arange(n, 0, -1, device="cuda", dtype=torch.int32)
    v = torch.stack([torch.arange(n, device="cuda"), -torch.arange(n, device="cuda")], dim=1)
    sk, sv = torch.ops.cusort.sort_pairs(x, v)
    ref = torch.sort(x, stable=True)
    assert torch.equal(sk, ref.values) and torch.equal(sv, v[ref.indices])
    assert torch.equal(torch.ops.cusort.argsort(x), ref.indices)
