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


def test_segmented_ops_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        k = torch.empty(1000, dtype=torch.int32, device="cuda")
        v = torch.empty(1000, 5, dtype=torch.int8, device="cuda")
        b = torch.empty(7, dtype=torch.int64, device="cuda")
        sk, sv = torch.ops.cusort.segmented_sort_pairs(k, v, b, b, True)
        assert sk.shape == k.shape and sv.shape == v.shape and sv.dtype == v.dtype
        assert torch.ops.cusort.segmented_sort_keys(k, b, b).shape == k.shape


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


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("row", [(3, torch.uint8), (6, torch.int32), (3, torch.int64), (2, torch.int64)])
@pytest.mark.parametrize("descending", [False, True])
def test_sort_pairs_any_payload_width(row, descending):
    # rows of 3, 24, 24 and 16 bytes: the odd widths take the permutation + gather path
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    n = 300_007
    x = torch.randint(-1000, 1000, (n,), device="cuda", dtype=torch.int32, generator=g)
    cols, dt = row
    v = torch.randint(-100, 100, (n, cols), device="cuda", generator=g).to(dt)
    ref = torch.sort(x, descending=descending, stable=True)
    sk, sv = torch.ops.cusort.sort_pairs(x, v, descending)
    assert torch.equal(sk, ref.values) and torch.equal(sv, v[ref.indices])


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("descending", [False, True])
def test_segmented_ops_match_per_segment_sort(descending):
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    n = 400_000
    x = torch.randint(-50, 50, (n,), device="cuda", dtype=torch.int64, generator=g)
    v = torch.arange(n, device="cuda", dtype=torch.int32)
    # lengths 0 .. ~60k (tiny, warp, CTA and multi-tile classes) with gaps between segments
    cuts, pos = [], 0
    lens = [0, 1, 17, 33, 300, 900, 4000, 9000, 60_000, 2, 70_000]
    for ln in lens:
        cuts.append((pos, pos + ln))
        pos += ln + 5
    b = torch.tensor([c[0] for c in cuts], dtype=torch.int64, device="cuda")
    e = torch.tensor([c[1] for c in cuts], dtype=torch.int64, device="cuda")
    sk, sv = torch.ops.cusort.segmented_sort_pairs(x, v, b, e, descending)
    ko = torch.ops.cusort.segmented_sort_keys(x, b, e, descending)
    inside = torch.zeros(n, dtype=torch.bool, device="cuda")
    for s0, s1 in cuts:
        inside[s0:s1] = True
        ref = torch.sort(x[s0:s1], descending=descending, stable=True)
        assert torch.equal(sk[s0:s1], ref.values) and torch.equal(ko[s0:s1], ref.values)
        assert torch.equal(sv[s0:s1], v[s0:s1][ref.indices])
    # positions outside every segment keep the input
    assert torch.equal(sk[~inside], x[~inside]) and torch.equal(sv[~inside], v[~inside])
    assert torch.equal(ko[~inside], x[~inside])
