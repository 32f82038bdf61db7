"""One rank of the two-GPU split-KV check (launched by tests/test_multi_gpu.py
through torch.distributed.run): the in-kernel peer exchange and the NCCL
all-gather path against a single-GPU decode over the whole context."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "llm-inference-webgpu_b200"))
import b2a  # noqa: E402
from b2a import dist as bd  # noqa: E402

H, KVH, D, THETA = 14, 2, 64, 1e6


class _CAI:
    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape, "typestr": "<f2", "version": 3}


def fill(cache, k, v):
    """k, v [batch, KVH, n, D] (one layer) or [batch, layers, KVH, n, D] f16 into
    positions 0..n-1."""
    if k.dim() == 4:
        k, v = k[:, None], v[:, None]
    layers = k.shape[1]
    kp, vp, _ = cache.pools()
    shape = (cache.batch, layers, KVH, cache.capacity, D)
    torch.as_tensor(_CAI(kp, shape), device=k.device)[:, :, :, :k.shape[3]].copy_(k)
    torch.as_tensor(_CAI(vp, shape), device=v.device)[:, :, :, :v.shape[3]].copy_(v)
    cache.setLengths([k.shape[3]] * cache.batch)


def multilayer(ctx, dev, rank, world, failures):
    """Three layers per call through one exchange: the peer path and the NCCL
    path against one single-GPU decode of all three layers."""
    batch, layers, total = 3, 3, 2100
    lo, hi = bd.position_slice(total, world, rank)
    g = torch.Generator(device=dev)
    g.manual_seed(6)
    kfull = torch.randn(batch, layers, KVH, total, D, generator=g, device=dev).half()
    vfull = torch.randn(batch, layers, KVH, total, D, generator=g, device=dev).half()
    q = torch.randn(batch, layers, H, D, generator=g, device=dev).half()
    kn = torch.randn(batch, layers, KVH, D, generator=g, device=dev).half()
    vn = torch.randn(batch, layers, KVH, D, generator=g, device=dev).half()
    pos = torch.full((batch,), total, dtype=torch.int32, device=dev)
    rope = b2a.RopeTable(ctx, D, THETA, total + 1)
    cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), hi - lo + 1, batch=batch, dtype="f16")
    fill(cache, kfull[:, :, :, lo:hi].contiguous(), vfull[:, :, :, lo:hi].contiguous())
    peer = bd.PeerSplitKV(ctx, cache, rope, 0, H, rank, world, num_layers=layers)
    out_peer = torch.empty(batch, layers, H, D, device=dev)
    for _ in range(3):
        peer.step(q, kn, vn, pos, out_peer)
    nccl = bd.cuda_split_kv(ctx, cache, rope, 0, H, rank, world, num_layers=layers)
    local = torch.empty(batch, layers, H, D + 4, device=dev)
    out_nccl = torch.empty(batch, layers, H, D, device=dev)
    nccl.step(q, kn, vn, pos, local, out_nccl)
    # the same step through one C-ABI call over this test's own NCCL communicator
    uid = bd.gather_handles(bd.NcclComm.unique_id(), world)[:bd.NcclComm.ID_BYTES]
    comm = bd.NcclComm(uid, world, rank)
    out_capi = torch.empty(batch, layers, H, D, device=dev)
    capi = bd.NcclSplitKV(ctx, cache, rope, 0, H, comm, num_layers=layers)
    for _ in range(2):
        capi.step(q, kn, vn, pos, out_capi)
    full = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), total + 1, batch=batch, dtype="f16")
    fill(full, kfull, vfull)
    out_full = torch.empty(batch, layers, H, D, device=dev)
    b2a.attentionDecode(ctx, full, rope, 0, q, kn, vn, out_full, H, numLayers=layers)
    ctx.synchronize()
    torch.cuda.synchronize(dev)
    d_peer = (out_peer - out_full).abs().max().item()
    d_nccl = (out_nccl - out_full).abs().max().item()
    d_capi = (out_capi - out_full).abs().max().item()
    if not d_peer <= 2e-3:
        failures.append(f"3-layer peer exchange off by {d_peer}")
    if not d_nccl <= 2e-3:
        failures.append(f"3-layer nccl path off by {d_nccl}")
    if not d_capi <= 2e-3:
        failures.append(f"3-layer C-ABI nccl call off by {d_capi}")
    if not torch.equal(out_capi, out_nccl):
        failures.append("C-ABI nccl call and the torch.distributed nccl path differ")
    comm.close()
    peer.close()
    return d_peer, d_nccl


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ctx = b2a.Context(rank)
    stream = torch.cuda.Stream(dev)
    ctx.set_stream(stream)
    batch, total = 4, 3000
    lo, hi = bd.position_slice(total, world, rank)
    failures = []
    with torch.cuda.stream(stream):
        g = torch.Generator(device=dev)
        g.manual_seed(5)
        kfull = torch.randn(batch, KVH, total, D, generator=g, device=dev).half()
        vfull = torch.randn(batch, KVH, total, D, generator=g, device=dev).half()
        q = torch.randn(batch, H, D, generator=g, device=dev).half()
        kn = torch.randn(batch, KVH, D, generator=g, device=dev).half()
        vn = torch.randn(batch, KVH, D, generator=g, device=dev).half()
        pos = torch.full((batch,), total, dtype=torch.int32, device=dev)
        rope = b2a.RopeTable(ctx, D, THETA, total + 1)
        cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(1, KVH, D, H), hi - lo + 1, batch=batch, dtype="f16")
        fill(cache, kfull[:, :, lo:hi].contiguous(), vfull[:, :, lo:hi].contiguous())
        peer = bd.PeerSplitKV(ctx, cache, rope, 0, H, rank, world)
        out_peer = torch.empty(batch, H, D, device=dev)
        for _ in range(4):   # both buffer parities, twice
            peer.step(q, kn, vn, pos, out_peer)
        nccl = bd.cuda_split_kv(ctx, cache, rope, 0, H, rank, world)
        local = torch.empty(batch, H, D + 4, device=dev)
        out_nccl = torch.empty(batch, H, D, device=dev)
        nccl.step(q, kn, vn, pos, local, out_nccl)
        full = b2a.GpuKVCache(ctx, b2a.CacheConfig(1, KVH, D, H), total + 1, batch=batch, dtype="f16")
        fill(full, kfull, vfull)
        out_full = torch.empty(batch, 1, H, D, device=dev)
        b2a.attentionDecode(ctx, full, rope, 0, q.view(batch, 1, H, D), kn.view(batch, 1, KVH, D),
                            vn.view(batch, 1, KVH, D), out_full, H)
    ctx.synchronize()
    torch.cuda.synchronize(dev)
    d_peer = (out_peer - out_full.view(batch, H, D)).abs().max().item()
    d_nccl = (out_nccl - out_full.view(batch, H, D)).abs().max().item()
    if not d_peer <= 2e-3:
        failures.append(f"peer exchange off by {d_peer}")
    if not d_nccl <= 2e-3:
        failures.append(f"nccl path off by {d_nccl}")
    with torch.cuda.stream(stream):
        m_peer, m_nccl = multilayer(ctx, dev, rank, world, failures)
    gathered = torch.empty(world, batch, H, D, device=dev)
    dist.all_gather_into_tensor(gathered.view(world * batch, H, D), out_peer)
    if not all(torch.equal(gathered[0], gathered[r]) for r in range(world)):
        failures.append("ranks disagree")
    print(f"rank {rank}: peer {d_peer:.2e} nccl {d_nccl:.2e} 3-layer peer {m_peer:.2e} nccl {m_nccl:.2e} "
          f"{'FAIL ' + '; '.join(failures) if failures else 'ok'}", flush=True)
    peer.close()
    dist.destroy_process_group()
    sys.exit(1 if failures else 0)


if __name__ == "__main__":
    main()
