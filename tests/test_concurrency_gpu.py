"""Concurrent callers on one device: several host threads, each with its own
CUDA stream, run chunked scans, full reductions and row argmaxes at the same
time through the public seams.  Every call keeps its scratch (workspace,
partials, tickets, scan status) per stream, so the results must equal the
oracle's exactly as when the calls run alone (the reference's CudaDevice is
Send + Sync and its calls may come from any thread)."""
import threading

import numpy as np
import pytest

from hephaestus_b200 import CudaAxisReductionOps, CudaFullReductionOps, CudaScanOps
from hephaestus_b200.core import CumSumOp, Layout, StridedView, SumOp

pytestmark = pytest.mark.gpu

THREADS = 4
ROUNDS = 3
SCAN_N = (1 << 23) + 1000  # long enough for the chunked (cooperative) scan kernel
SUM_N = (1 << 20) + 3
ROWS, COLS = 64, 4096


def test_threads_on_separate_streams(device, oracle):
    import torch

    work = []
    for t in range(THREADS):
        xs = oracle.generate(oracle.GEN_U32_LOW4, 10 + t, SCAN_N)
        xf = oracle.generate(oracle.GEN_F32_UNIFORM_PM1, 20 + t, SUM_N)
        xm = oracle.generate(oracle.GEN_F32_NORMAL, 30 + t, ROWS * COLS)
        work.append(dict(
            xs=device.upload(xs), ys=device.alloc_zeroed(np.uint32, SCAN_N),
            want_s=oracle.scan_axis(xs, [SCAN_N], 0, exclusive=(t % 2 == 0)), excl=(t % 2 == 0),
            xf=device.upload(xf), yf=device.alloc_zeroed(np.float32, 1),
            want_f=float(oracle.reduce_full(xf, [SUM_N])), tol_f=1e-5 * float(np.abs(xf).sum()),
            xm=device.upload(xm), vals=device.alloc_zeroed(np.float32, ROWS),
            idx=device.alloc_zeroed(np.uint32, ROWS), want_i=oracle.arg_reduce_axis(xm, [ROWS, COLS], 1)[1],
            stream=torch.cuda.Stream(device=0)))
    device.synchronize()
    errors = []
    start = threading.Barrier(THREADS)

    def run(t):
        w = work[t]
        sp = w["stream"].cuda_stream
        scans, fulls, axes = CudaScanOps(), CudaFullReductionOps(), CudaAxisReductionOps()
        ls, ol = Layout.c_contiguous([SCAN_N]), Layout.c_contiguous([ROWS, 1])
        try:
            start.wait()
            for r in range(ROUNDS):
                scans.scan_axis_into(CumSumOp, device, StridedView(w["xs"], ls), 0, 0, StridedView(w["ys"], ls),
                                     exclusive=w["excl"], stream=sp)
                fulls.reduce_full_into(SumOp, device, StridedView(w["xf"], Layout.c_contiguous([SUM_N])),
                                       StridedView(w["yf"], Layout.c_contiguous([1])), stream=sp)
                axes.argmax_axis_into(device, StridedView(w["xm"], Layout.c_contiguous([ROWS, COLS])), 1,
                                      StridedView(w["vals"], ol), StridedView(w["idx"], ol), stream=sp)
                device.synchronize_stream(sp)
                got_s = device.download_owned(w["ys"])
                if not np.array_equal(got_s, w["want_s"]):
                    errors.append(f"thread {t} round {r}: scan differs at {np.flatnonzero(got_s != w['want_s'])[:4]}")
                got_f = float(device.download_owned(w["yf"])[0])
                if abs(got_f - w["want_f"]) > w["tol_f"]:
                    errors.append(f"thread {t} round {r}: sum {got_f} vs {w['want_f']}")
                if not np.array_equal(device.download_owned(w["idx"]), w["want_i"]):
                    errors.append(f"thread {t} round {r}: argmax indices differ")
        except Exception as e:  # noqa: BLE001 - reported below with the thread id
            errors.append(f"thread {t}: {type(e).__name__}: {e}")

    threads = [threading.Thread(target=run, args=(t,)) for t in range(THREADS)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not any(th.is_alive() for th in threads), "a worker thread did not finish"
    assert not errors, "\n".join(errors)
    device.synchronize()


def test_concurrent_device_acquisition(oracle):
    """Sixteen threads open the same ordinal at once (the reference's
    concurrency test does the same for CudaDevice acquisition) and each runs a
    reduction through its own handle."""
    from hephaestus_b200 import CudaDevice

    x = oracle.generate(oracle.GEN_U32_LOW4, 5, 100_003)
    want = int(x.astype(np.uint64).sum() & 0xffffffff)
    got, errors = [None] * 16, []
    start = threading.Barrier(16)

    def run(t):
        try:
            start.wait()
            dev = CudaDevice(0)
            buf, out = dev.upload(x), dev.alloc_zeroed(np.uint32, 1)
            CudaFullReductionOps().reduce_full_into(SumOp, dev, StridedView(buf, Layout.c_contiguous([x.size])),
                                                    StridedView(out, Layout.c_contiguous([1])))
            got[t] = int(dev.download_owned(out)[0])
        except Exception as e:  # noqa: BLE001 - reported below with the thread id
            errors.append(f"thread {t}: {type(e).__name__}: {e}")

    threads = [threading.Thread(target=run, args=(t,)) for t in range(16)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not errors, "\n".join(errors)
    assert got == [want] * 16
