"""torch.ops registration (fufft_b200.torch_ops): the ops exist with the
documented schemas and their fake implementations give the right shapes
without a GPU; on a GPU each op equals the direct fufft_b200.ops call."""
import numpy as np
import pytest
import torch


def test_ops_registered_with_fake_shapes():
    import fufft_b200.torch_ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    for name in ("conv", "conv2d", "c2c", "filter_from_taps"):
        assert hasattr(torch.ops.fufft, name)
    with FakeTensorMode():
        a = torch.empty(8, 4096, dtype=torch.complex64)
        assert torch.ops.fufft.conv(a, a, 4096, 3, 1, 4096).shape == a.shape
        assert torch.ops.fufft.c2c(a, 4096, -1).shape == a.shape
        assert torch.ops.fufft.filter_from_taps(a, 4096, 3).shape == a.shape
        img = torch.empty(2, 64, 64, dtype=torch.complex64)
        assert torch.ops.fufft.conv2d(img, img[0], 64, 64, 3, 1, 0).shape == img.shape


@pytest.mark.gpu
def test_ops_match_direct_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import fufft_b200.torch_ops  # noqa: F401
    from fufft_b200 import ops
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    n = 4096
    a = torch.randn(6, n, dtype=torch.complex64, device="cuda", generator=g)
    taps = torch.randn(6, n, dtype=torch.complex64, device="cuda", generator=g)
    b = torch.ops.fufft.filter_from_taps(taps, n, ops.LAYOUT_R16_BPERM)
    assert torch.equal(b.view(-1), ops.filter_from_taps(taps.view(-1), n, ops.LAYOUT_R16_BPERM))
    got = torch.ops.fufft.conv(a, b, n, ops.LAYOUT_R16_BPERM, ops.MID_MULTIPLY, n)
    assert torch.equal(got.view(-1), ops.conv(a.view(-1), b.view(-1), n, ops.LAYOUT_R16_BPERM))
    spec = torch.ops.fufft.c2c(a, n, -1)
    ref = torch.fft.fft(a.to(torch.complex128), dim=1)
    assert float((spec - ref).abs().pow(2).sum() / ref.abs().pow(2).sum()) ** 0.5 < 2e-6
    # traceable as one graph node (dynamo + AOT autograd, eager kernels: no code generation)
    f = torch.compile(lambda x, y: torch.ops.fufft.conv(x, y, n, ops.LAYOUT_R16_BPERM, ops.MID_MULTIPLY, n),
                      fullgraph=True, backend="aot_eager")
    assert torch.equal(f(a, b), got)
