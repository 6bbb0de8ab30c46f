"""Worker for test_gather_mgpu.py (run under torchrun, one process per GPU):
column-sharded GEMMs whose panels are gathered into every rank's full C by
b2b_{h,s,d}gemm_gather, checked against the CPU oracle on every rank.  Exits
non-zero on any mismatch."""
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "cublas-rs_b200"))
sys.path.insert(0, os.path.join(HERE, ".."))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import b2blas  # noqa: E402
from b2blas import shard  # noqa: E402
from oracle import oracle  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    h = b2blas.Handle(local)
    failures = []
    cases = [("h", 640, 1000, 384, 1.0, 0.0), ("h", 1024, 3072, 512, 0.5, 0.0), ("h", 300, 776, 200, 1.0, 0.5),
             ("s", 257, 1000, 130, 1.5, 0.0), ("s", 300, 520, 64, 1.5, 0.5), ("d", 200, 264, 96, 1.25, -0.5)]
    for prec, m, n_total, k, alpha, beta in cases:
        widths = shard.column_panels(n_total, world, 8)
        c0 = sum(widths[:rank])
        w = widths[rank]
        if prec == "h":
            A = oracle.normal_f16(m * k, 5, 1, 0.0, 0.1)
            B = oracle.normal_f16(k * n_total, 5, 2, 0.0, 0.1)
            C0 = oracle.normal_f16(m * n_total, 5, 3, 0.0, 0.1)
            dt, ref = np.uint16, oracle.hgemm_f64(m, n_total, k, alpha, A, B, beta, C0)
            tol = 2e-2
        else:
            f = oracle.uniform_f32 if prec == "s" else oracle.uniform_f64
            A, B, C0 = f(m * k, 5, 1), f(k * n_total, 5, 2), f(m * n_total, 5, 3)
            dt = np.float32 if prec == "s" else np.float64
            ref = (oracle.sgemm_f64 if prec == "s" else oracle.dgemm_f64)(m, n_total, k, alpha, A, B, beta, C0)
            tol = oracle.tol_normwise(k, "f32" if prec == "s" else "f64")
        bpanel = shard.panel_of(B, k, n_total, c0, c0 + w)
        peers = shard.PeerBuffers(h, m * n_total, dt)
        # Own buffer: NaN everywhere (must all be overwritten) except, when
        # beta != 0, this rank's input panel.
        init = np.full(m * n_total, 0x7E00, np.uint16) if prec == "h" else np.full(m * n_total, np.nan, dt)
        if beta != 0.0:
            init.reshape(m, n_total)[:, c0:c0 + w] = C0.reshape(m, n_total)[:, c0:c0 + w]
        b2blas_lib = b2blas.load_library()
        import ctypes

        b2blas_lib.b2b_memcpy_h2d(h._h, ctypes.c_void_p(peers.buf.ptr), ctypes.c_void_p(init.ctypes.data), init.nbytes)
        h.synchronize()
        dist.barrier()
        a, b = h.upload(A), h.upload(bpanel)
        cfg = b2blas.GemmConfig(m, w, k, alpha, beta)
        getattr(h, f"{prec}gemm_gather")(cfg, a, b, n_total, c0, peers.ptrs, rank)
        h.synchronize()
        dist.barrier()
        got = h.download(peers.buf)
        err = oracle.rel_err(got, ref)
        if not err <= tol:
            failures.append(f"{prec} {m}x{n_total}x{k} beta={beta}: rel err {err:.3e} > {tol:.1e}")
        # every rank holds the same bits
        sig = torch.tensor([int(np.frombuffer(got.tobytes(), np.uint8)[::97].astype(np.int64).sum())],
                           device="cuda", dtype=torch.int64)
        lo, hi = sig.clone(), sig.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        if lo.item() != hi.item():
            failures.append(f"{prec} {m}x{n_total}x{k}: ranks differ")
        peers.close()
        a.free()
        b.free()
    h.close()
    dist.destroy_process_group()
    for f in failures:
        print(f"rank {rank}: FAIL {f}", flush=True)
    if not failures:
        print(f"rank {rank}: all gather cases OK", flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
