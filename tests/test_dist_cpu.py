"""The multi-rank decode orchestration on CPU: position slicing, sequence
partitioning, and a world-size-2 gloo run of the split-KV step whose compute is
the CPU oracle (the CUDA kernels run the same step on GPUs; see
tests/test_gpu_parity.py::test_split_kv_partials_combine_to_full_decode)."""
import datetime
import math
import os
import socket
import sys

import numpy as np
import pytest

from b2a import dist as bd

LOG2E = 1.0 / math.log(2.0)
RENDEZVOUS_S = 90    # ranks joining (each spawned child imports torch first)
COLLECTIVE_S = 5     # one collective of the step: a missing rank must fail it quickly


def test_position_slices_partition_the_sequence():
    for total in (1, 7, 32768, 32769):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                lo, hi = bd.position_slice(total, world, r)
                assert 0 <= lo <= hi <= total
                covered.extend(range(lo, hi))
            assert covered == list(range(total))
    with pytest.raises(ValueError):
        bd.position_slice(10, 2, 2)


def test_lpt_partition_is_balanced_and_deterministic():
    rng = np.random.default_rng(1234)
    w = [int(x) for x in rng.integers(256, 4097, size=64)]
    for world in (1, 2, 4, 8):
        bins = bd.lpt_partition(w, world)
        assert sorted(i for b in bins for i in b) == list(range(64))
        loads = [sum(w[i] for i in b) for b in bins]
        assert max(loads) - min(loads) <= max(w)
        assert bins == bd.lpt_partition(w, world)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_partial(oracle, q, kh, vh, lo, hi, n_heads, group, head_dim):
    """The product's partial format from the CPU oracle: [heads, D+4] with the
    unnormalised output, then m in base-2 units and l."""
    out = np.zeros((n_heads, head_dim + 4), np.float32)
    for h in range(n_heads):
        g = h // group
        if hi <= lo:
            out[h, head_dim] = -np.inf
            continue
        m, l, o = oracle.decode_partial(q[h], kh[g], vh[g], lo, hi, head_dim)
        out[h, :head_dim] = o
        out[h, head_dim] = m * LOG2E
        out[h, head_dim + 1] = l
    return out


def _combine(stacked, head_dim):
    """The product's combine (k_combine) restated: ascending parts, base 2."""
    m = stacked[..., head_dim]
    l = stacked[..., head_dim + 1]
    valid = l > 0
    mx = np.where(valid, m, -np.inf).max(axis=0)
    w = np.where(valid, np.exp2(m - mx), 0.0)
    num = (w[..., None] * stacked[..., :head_dim]).sum(axis=0)
    return (num / (w * l).sum(axis=0)[..., None]).astype(np.float32)


def _worker(rank, world, port, q, kh, vh, total, drop_rank, result_path):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "llm-inference-webgpu_b200"))
    from oracle import oracle
    from b2a import dist as bdist

    # the rendezvous includes every spawned rank importing torch, which can take
    # tens of seconds on a loaded machine: give it a generous limit, and bound
    # the step's collective separately with a group of its own
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=RENDEZVOUS_S))
    step_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=COLLECTIVE_S))
    heads, group, head_dim = q.shape[0], q.shape[0] // kh.shape[0], q.shape[1]
    lo, hi = bdist.position_slice(total, world, rank)

    def partial_fn(qq, k_new, v_new, positions, out_partial):
        out_partial[...] = torch.from_numpy(_oracle_partial(oracle, qq, kh, vh, lo, hi, heads, group, head_dim))

    def gather_fn(local):
        if rank == drop_rank:
            raise SystemExit(0)   # this rank leaves between steps, before the collective
        flat = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype)
        dist.all_gather_into_tensor(flat, local, group=step_group)
        return flat.view((world,) + tuple(local.shape))

    def combine_fn(stacked, out):
        out[...] = torch.from_numpy(_combine(stacked.numpy(), head_dim))

    step = bdist.SplitKVDecode(rank, world, partial_fn, gather_fn, combine_fn)
    local = torch.zeros(heads, head_dim + 4)
    out = torch.zeros(heads, head_dim)
    try:
        step.step(q, None, None, None, local, out)
        np.save(result_path, out.numpy())
    except Exception as e:   # the surviving rank: the collective must fail, not hang
        with open(result_path + ".err", "w") as f:
            f.write(type(e).__name__ + ": " + str(e)[:200])
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, drop_rank, tmp_path, oracle):
    import multiprocessing as mp
    heads, kvh, hd, total = 14, 2, 64, 301
    q = oracle.normal_array(heads * hd, 3).reshape(heads, hd)
    kh = oracle.normal_array(kvh * total * hd, 4).reshape(kvh, total, hd)
    vh = oracle.normal_array(kvh * total * hd, 5).reshape(kvh, total, hd)
    ctx = mp.get_context("spawn")
    port = _free_port()
    paths = [str(tmp_path / f"rank{r}.npy") for r in range(world)]
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, kh, vh, total, drop_rank, paths[r]))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank did not finish: the split-KV step hung")
    return q, kh, vh, total, paths


def test_split_kv_step_two_ranks_gloo(tmp_path, oracle):
    q, kh, vh, total, paths = _run(2, -1, tmp_path, oracle)
    outs = [np.load(p) for p in paths]
    assert np.array_equal(outs[0], outs[1]), "ranks must agree bit for bit"
    heads, hd = q.shape
    ref = np.stack([oracle.grouped_attention(q[h], kh[h // 7].reshape(-1), vh[h // 7].reshape(-1), 1, total - 1,
                                             1, 1, hd) for h in range(heads)])
    assert np.abs(outs[0] - ref).max() < 1e-5


def test_split_kv_step_missing_rank_fails_fast(tmp_path, oracle):
    """A rank that leaves before the gather: the other rank's collective ends
    with an error within the step group's timeout instead of hanging."""
    import time
    t0 = time.monotonic()
    _, _, _, _, paths = _run(2, 1, tmp_path, oracle)
    assert os.path.exists(paths[0] + ".err"), "rank 0 should have seen the collective fail"
    assert not os.path.exists(paths[0])
    # spawn + rendezvous + the bounded collective, far below the rendezvous limit
    assert time.monotonic() - t0 < RENDEZVOUS_S


def _handle_worker(rank, world, port, result_path):
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "llm-inference-webgpu_b200"))
    from b2a import dist as bdist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=RENDEZVOUS_S))
    try:
        got = bdist.gather_handles(bytes([rank + 1]) * 64, world)
        with open(result_path, "wb") as f:
            f.write(got)
    finally:
        dist.destroy_process_group()


def test_exchange_handles_gathered_in_rank_order(tmp_path):
    """PeerSplitKV's setup step: every rank's 64-byte exchange handle reaches
    every rank, in rank order (gloo on CPU; NCCL on GPUs)."""
    import multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    paths = [str(tmp_path / f"h{r}.bin") for r in range(world)]
    procs = [ctx.Process(target=_handle_worker, args=(r, world, port, paths[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            raise AssertionError("handle exchange hung")
    want = bytes([1]) * 64 + bytes([2]) * 64
    for path in paths:
        with open(path, "rb") as f:
            assert f.read() == want
