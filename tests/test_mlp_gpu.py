"""The mlp example's forward as bench.py runs it: 4 layers 1024-4096-4096-4096-1024,
batch 4096, bias (+ReLU on hidden layers) fused into the SGEMM epilogue.  Two
half-batch streams must give the bits of one stream, and both must match a
PyTorch fp64 forward of the same weights within the FP32 GEMM bound."""
import pytest

pytestmark = pytest.mark.gpu


class _Args:
    fused = True
    tf32x3 = False

    def __init__(self, streams):
        self.mlp_streams = streams


def test_mlp_two_streams_same_bits_and_fp32_reference():
    import torch

    import b2blas
    import bench

    outs, w1 = [], None
    for streams in (1, 2):
        s = torch.cuda.Stream()
        torch.cuda.set_stream(s)
        h = b2blas.Handle(0)
        h.set_stream(s.cuda_stream)
        try:
            w = bench.MlpWorkload(h, 0, 1, _Args(streams))
            w.step()
            torch.cuda.synchronize()
            outs.append(w.Z[-1].clone())
            if streams == 1:
                w1 = w
            else:
                w.close()
        finally:
            h.set_stream(None)
            h.close()
    torch.cuda.set_stream(torch.cuda.default_stream())
    assert torch.equal(outs[0], outs[1])
    x = w1.X.double()
    for i in range(4):
        x = x @ w1.W[i].double() + w1.bias_vec[i].double()
        if i < 3:
            x = torch.relu(x)
    err = ((outs[0].double() - x).norm() / x.norm()).item()
    assert err <= 4 * 4096 * 2.0 ** -24, err  # 4*K*eps32 for the widest layer
