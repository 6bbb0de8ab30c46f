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
    # The HGEMM gather through an NVLink multicast object (torch symmetric
    # memory binds one buffer per rank and maps the multicast address).
    try:
        import torch.distributed._symmetric_memory as symm
        have_symm = True
    except Exception:  # noqa: BLE001 -- older torch: nothing to test
        have_symm = False
    if have_symm:
        for m, n_total, k, alpha in ((640, 1000, 384, 1.0), (1024, 3072, 512, 0.5)):
            widths = shard.column_panels(n_total, world, 8)
            c0, w = sum(widths[:rank]), widths[rank]
            A = oracle.normal_f16(m * k, 7, 1, 0.0, 0.1)
            B = oracle.normal_f16(k * n_total, 7, 2, 0.0, 0.1)
            ref = oracle.hgemm_f64(m, n_total, k, alpha, A, B)
            t = symm.empty(m * n_total, dtype=torch.float16, device=f"cuda:{local}")
            hd = symm.rendezvous(t, dist.group.WORLD.group_name)
            mc = int(getattr(hd, "multicast_ptr", 0) or 0)
            ok_mc = torch.tensor([1 if mc else 0], device="cuda")
            dist.all_reduce(ok_mc, op=dist.ReduceOp.MIN)
            if ok_mc.item():
                t.view(torch.int16).fill_(0x7E00)  # NaN: every element must be written
                torch.cuda.synchronize()
                dist.barrier()
                a, b = h.upload(A), h.upload(shard.panel_of(B, k, n_total, c0, c0 + w))
                try:
                    h.hgemm_gather_multicast(b2blas.GemmConfig(m, w, k, alpha, 0.0), a, b, n_total, c0, mc,
                                             t.data_ptr())
                except b2blas.CublasError as e:
                    failures.append(f"multicast {m}x{n_total}x{k}: {e}")
                h.synchronize()
                dist.barrier()
                got = t.cpu().numpy().view(np.uint16)
                err = oracle.rel_err(got, ref)
                if not err <= 2e-2:
                    failures.append(f"multicast {m}x{n_total}x{k}: rel err {err:.3e}")
                a.free()
                b.free()
            else:
                print(f"rank {rank}: no multicast address, multicast case skipped", flush=True)
            dist.barrier()
            del t, hd
    h.close()
    dist.barrier()
    dist.destroy_process_group()
    for f in failures:
        print(f"rank {rank}: FAIL {f}", flush=True)
    if not failures:
        print(f"rank {rank}: all gather cases OK", flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
