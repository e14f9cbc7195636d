"""Failure detection, exercised without faulting or hanging a GPU.

* Device side: every wait of the kernels on an mbarrier, flag or peer is
  bounded; on expiry the kernel records a ROLA_DEV_* code and returns.  The
  library's self-test makes such a wait run out (an mbarrier nothing
  completes, a 0.2 s limit) and the host reads the code; the context stays
  usable for the next forward.
* Host side (CPU, gloo): when a rank of the sequence-parallel group dies
  between layers, the surviving ranks' next exchange ends with an error within
  the process group's short timeout instead of waiting for ever.
"""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

ROLA_DEV_TIMEOUT_LOAD = 1


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_reports():
    from sparkdiffusion_b200 import _lib, ops

    _lib.load_library()
    assert _lib.device_status() == 0
    t0 = time.perf_counter()
    _lib.call("rola_b200_check_wait_timeout", 200000, torch.cuda.current_stream().cuda_stream)
    assert time.perf_counter() - t0 < 10.0
    assert _lib.device_status() == ROLA_DEV_TIMEOUT_LOAD  # read and cleared
    assert _lib.device_status() == 0
    # the context is still usable: a GEMM through the library afterwards
    x = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    w = (torch.randn(512, 512, device="cuda") * 0.05).to(torch.bfloat16)
    y = ops.qkv_gemm(x, w)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    torch.testing.assert_close(y.float(), (x.float() @ w.float().t()), rtol=2e-2, atol=2e-2)


def test_wait_timeout_argument_checked_without_launch():
    from sparkdiffusion_b200 import _lib

    _lib.load_library()
    with pytest.raises(ValueError, match="limit_us"):
        _lib.call("rola_b200_check_wait_timeout", 0, None)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, result_dir, mode):
    import torch.distributed as dist

    from sparkdiffusion_b200.ulysses import head_to_seq, seq_to_head

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    B, p, Ls, X = 1, world, 6, 4
    send = torch.arange(B * p * Ls * X, dtype=torch.float32).view(B, p, Ls, X) + 100 * rank
    seq_to_head(send)  # layer 1: every rank takes part
    if rank == world - 1:
        if mode == "stall":
            time.sleep(25)  # this rank stops answering between layers ...
        os._exit(0)  # ... or dies, without a word to the others
    t0 = time.perf_counter()
    err = ""
    try:
        recv, _ = seq_to_head(send)  # layer 2: the exchange must fail, not hang
        head_to_seq(recv.view(B, p * Ls, X), p)
    except Exception as e:  # noqa: BLE001 - the failure is what is being checked
        err = type(e).__name__ + ": " + str(e)[:200]
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{time.perf_counter() - t0:.2f}\n{err}\n")
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_lost_rank_turns_next_exchange_into_error(tmp_path, mode):
    """A rank exits (its sockets close: the survivor sees it at once) or stalls
    (the survivor gives up at the process group's 5 s timeout)."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, world, port, str(tmp_path), mode)) for r in range(world)]
    for pr in procs:
        pr.start()
    procs[0].join(timeout=60)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    if not (tmp_path / "rank0.txt").exists():
        pytest.fail("the surviving rank did not give up within 60 s")
    with open(tmp_path / "rank0.txt") as f:
        elapsed, err = f.read().split("\n", 1)
    assert err.strip(), "the survivor's exchange with a dead rank did not raise"
    assert float(elapsed) < 20.0, f"gave up only after {elapsed} s"

