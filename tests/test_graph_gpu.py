"""The library's device-buffer calls inside a CUDA graph.

Every launch path is capturable once the call's workspace and one-time
setup (kernel attributes, occupancy queries) exist, so a step is captured
after one eager call of the same shapes.  The graph's replays must give the
eager results bit for bit (the kernels are deterministic)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_capture_and_replay(oracle):
    import torch

    import b2blas

    h = b2blas.Handle(0)
    s = torch.cuda.Stream()
    try:
        h.set_stream(s.cuda_stream)
        m = n = k = 1024
        A = oracle.normal_f16(m * k, 70, 1, 0.0, 0.1)
        B = oracle.normal_f16(k * n, 70, 2, 0.0, 0.1)
        a16, b16, c16 = h.upload(A), h.upload(B), h.zeroed(m * n, np.uint16)
        cfg = b2blas.GemmConfig(m, n, k, 1.0, 0.0)
        gm, gn = 4096, 2048
        G = oracle.uniform_f32(gm * gn, 70, 3)
        x = oracle.uniform_f32(gm, 70, 4)
        g, xd, yd = h.upload(G), h.upload(x), h.zeroed(gn)
        dot = h.zeroed(1)

        def step():
            h.hgemm(cfg, a16, b16, c16)
            h.sgemv(1, gm, gn, 1.0, g, xd, 0.0, yd)  # T: split-row partials in workspace
            h.sreduce_async(b2blas.Handle.ReduceOp.Dot, gn, yd, yd, dot)

        with torch.cuda.stream(s):
            step()  # eager: sizes the workspace, sets kernel attributes
        h.synchronize()
        eager = (h.download(c16), h.download(yd), h.download(dot))

        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step()
        with torch.cuda.stream(s):
            for _ in range(3):
                h.memset(yd, 0)  # the replay recomputes y and the dot from scratch
                graph.replay()
        s.synchronize()
        replayed = (h.download(c16), h.download(yd), h.download(dot))
        for e, r in zip(eager, replayed):
            assert np.array_equal(e, r)
        ref = oracle.sgemv_f64(1, gm, gn, 1.0, G, x, 0.0, np.zeros(gn, np.float32))
        assert oracle.rel_err(replayed[1], ref) <= oracle.tol_normwise(gm, "f32")
        del graph
    finally:
        h.set_stream(None)
        h.close()
