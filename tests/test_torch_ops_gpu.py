"""torch boundary (hephaestus_b200.torch_ops) against torch's own ops on CUDA
tensors: integers exact, floats within 1e-5 * sum|x| (f32)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_torch_ops_match_torch():
    import torch
    import hephaestus_b200.torch_ops as T
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.rand(513, 1027, device="cuda", generator=g) * 2 - 1
    tol = 1e-5 * float(x.abs().sum())
    assert abs(float(T.sum(x)) - float(x.double().sum())) <= tol
    assert float(T.max(x)) == float(x.max()) and float(T.min(x)) == float(x.min())
    assert abs(float(T.mean(x)) - float(x.double().mean())) <= tol / x.numel()
    for axis in (0, 1):
        assert torch.allclose(T.sum_axis(x, axis).double(), x.double().sum(axis, keepdim=True), atol=1e-3)
        assert torch.equal(T.max_axis(x, axis), x.max(axis, keepdim=True).values)
        v, i = T.argmax_axis(x, axis)
        assert torch.equal(i, x.argmax(axis, keepdim=True))
    xt = x.t()  # strided view
    assert torch.allclose(T.sum_axis(xt, 1).double(), xt.double().sum(1, keepdim=True), atol=1e-3)
    ints = torch.randint(-1000, 1000, (3_000_001,), device="cuda", dtype=torch.int32, generator=g)
    assert torch.equal(T.cumsum(ints), torch.cumsum(ints, 0, dtype=torch.int32))
    ex = T.cumsum(ints, exclusive=True)
    assert int(ex[0]) == 0 and torch.equal(ex[1:], torch.cumsum(ints, 0, dtype=torch.int32)[:-1])
    rev = T.cumsum(ints, reverse=True)
    assert torch.equal(rev, torch.flip(torch.cumsum(torch.flip(ints, [0]), 0, dtype=torch.int32), [0]))
    m = ints[:3_000_000].reshape(1000, 3000)[:, :2999]  # rows with a stride of 3000
    assert torch.equal(T.cumsum(m, axis=1), torch.cumsum(m, 1, dtype=torch.int32))
    a, b = x.flatten(), torch.flip(x.flatten(), [0])
    assert abs(float(T.dot(a, b)) - float((a.double() * b.double()).sum())) <= 1e-5 * float((a * b).abs().sum())
    assert abs(float(T.norm_l2(a)) - float(a.double().norm())) <= 1e-5 * float(a.double().norm())
    assert float(T.norm_max(a)) == float(a.abs().max())
