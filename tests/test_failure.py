"""Failure detection without a GPU fault.

* On the host (two `gloo` ranks on CPU, the column split's host logic): a rank that leaves
  between steps ends the other rank's next gather with an error, and a rank that never joins
  ends the first rank's set-up with an error, each within the process group's short timeout,
  not a hang.
* On the GPU: a gathered-output wait whose counter nothing will ever set (msq_wait_gathered
  with `produced` ahead of `arrivals`) gives up after the wait budget (msq_set_wait_budget, here
  50 ms instead of 2 s), and msq_device_status reports MSQ_E_TIMEOUT; the context stays usable
  and the next MatMulNBits is correct.
"""
import datetime
import json
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from modelsharp_b200 import synth
from modelsharp_b200.nsplit import ShardedMatMulNBits

TIMEOUT_S = 5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sharded(c):
    from oracle import oracle

    def local(a2, n0, n1):
        s = dict(c, b=c["b"][n0:n1], scales=np.asarray(c["scales"]).reshape(c["N"], -1)[n0:n1],
                 zp=c["zp"][n0:n1], N=n1 - n0, a=a2.numpy(), M=a2.shape[0])
        return torch.from_numpy(oracle.managed(s))

    return ShardedMatMulNBits(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, c["block_size"], align=16, local=local)


def _leaver(rank: int, world: int, port: int, out_dir: str):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=TIMEOUT_S))
    c = synth.make_case(81, 1, 256, 128, 4, 32, "packed")
    op = _sharded(c)
    a = torch.from_numpy(c["a"])
    op(a)  # step 1: both ranks
    if rank == 1:
        os._exit(0)  # leaves between steps: nothing of it is in flight
    t0 = time.monotonic()
    err = None
    try:
        op(a)  # step 2: the peer is gone
    except Exception as e:  # noqa: BLE001 -- any error, as long as it is not a hang
        err = type(e).__name__
    with open(os.path.join(out_dir, "rank0.json"), "w") as f:
        json.dump({"error": err, "seconds": time.monotonic() - t0}, f)
    os._exit(0)


def test_rank_leaving_between_steps_ends_the_next_gather_with_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    res = json.loads((tmp_path / "rank0.json").read_text())
    assert res["error"] is not None, res
    assert res["seconds"] < 6 * TIMEOUT_S, res


def _lonely(port: int, out_dir: str):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    t0 = time.monotonic()
    err = None
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=TIMEOUT_S))
    except Exception as e:  # noqa: BLE001
        err = type(e).__name__
    with open(os.path.join(out_dir, "lonely.json"), "w") as f:
        json.dump({"error": err, "seconds": time.monotonic() - t0}, f)
    os._exit(0)


def test_rank_that_never_joins_ends_set_up_with_an_error(tmp_path):
    p = mp.get_context("spawn").Process(target=_lonely, args=(_free_port(), str(tmp_path)))
    p.start()
    p.join(timeout=120)
    if p.is_alive():
        p.kill()
        pytest.fail("the rank waiting for a peer that never joins hung")
    res = json.loads((tmp_path / "lonely.json").read_text())
    assert res["error"] is not None, res
    assert res["seconds"] < 6 * TIMEOUT_S, res


@pytest.mark.gpu
def test_gathered_wait_that_never_completes_reports_timeout(cuda_device, native_lib):
    import ctypes as C

    from modelsharp_b200 import QuantizedWeights
    from modelsharp_b200 import _native as N
    from modelsharp_b200.weights import current_stream_ptr
    from oracle import oracle

    ctrl = torch.zeros(2, dtype=torch.int64, device=cuda_device)  # arrivals 0, produced 1: never met
    ctrl[1] = 1
    wt = N.WaitT()
    wt.arrivals, wt.produced, wt.nranks = ctrl.data_ptr(), ctrl.data_ptr() + 8, 1
    st = current_stream_ptr(cuda_device)
    torch.cuda.synchronize(cuda_device)
    assert N.lib().msq_device_status(None, st) == N.MSQ_OK  # nothing pending from earlier tests
    N.check(N.lib().msq_set_wait_budget(None, 50_000_000), "msq_set_wait_budget")  # 50 ms
    try:
        t0 = time.monotonic()
        N.check(N.lib().msq_wait_gathered(None, st, C.byref(wt)), "msq_wait_gathered")
        rc = N.lib().msq_device_status(None, st)
        dt = time.monotonic() - t0
    finally:
        N.check(N.lib().msq_set_wait_budget(None, 0), "msq_set_wait_budget")
    assert rc == N.MSQ_E_TIMEOUT, (rc, N.last_error())
    assert "gathered" in N.last_error() or "rank" in N.last_error(), N.last_error()
    assert dt < 1.5, dt  # well inside the default 2 s: the short budget was in force
    assert N.lib().msq_device_status(None, st) == N.MSQ_OK  # the flag was cleared
    # the context is still usable
    c = synth.make_case(82, 1, 512, 1024, 4, 128, "packed")
    w = QuantizedWeights(c["b"], c["scales"], c["zp"], 512, 1024, 4, 128, device=cuda_device)
    y = w.matmul(torch.from_numpy(c["a"]).to(cuda_device)).cpu().numpy()
    assert oracle.rel_l2(y, oracle.managed(c)) <= 1e-5
    w.free()
