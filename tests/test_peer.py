"""PeerSumNorm / cq_peer_sum_norm: the tensor-parallel row sum over NVLink
peer memory fused with the residual add and RMSNorm (csrc/cq_peer.cu).

On two GPUs: x must equal, bit for bit, the torch restatement (every rank's
part gathered, summed in fp32 in rank order, rounded to bf16, added to x with
one rounding); y within two bf16 ulps of the torch RMSNorm expression (the
fp32 sum of squares is reduced in another order, which can move the rounded
x * rsqrt(...) by one ulp, and the product with w rounds once more).  Eager calls alternate the
part buffers; a captured graph of four calls replays with new parts.  A
second case leaves one rank out: the other's bounded wait gives up and
cq_device_error reports 9 without the output being written."""

import multiprocessing as mp
import socket

import pytest
import torch

import _dist_workers as W


def _port():
    sk = socket.socket()
    sk.bind(("127.0.0.1", 0))
    port = sk.getsockname()[1]
    sk.close()
    return port


def _run(target, world, *args, timeout=240):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=timeout) for _ in range(world)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.gpu
@pytest.mark.parametrize("rows,dim", [(32, 4096), (1, 4096), (3, 1000)])
def test_peer_sum_norm_matches_torch(rows, dim):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _run(W.peer_sum_worker, 2, rows, dim)
    for rank, worst, code, err in res:
        assert err is None, err
        assert worst[0] == 0, worst  # x: bit-exact
        assert worst[1] <= 2, worst  # y: within two ulps
        assert code == 0


@pytest.mark.gpu
def test_peer_wait_gives_up_without_a_peer():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _run(W.peer_timeout_worker, 2)
    for rank, code, err in res:
        assert err is None, err
    assert res[0][1] == (9, True), res[0][1]
