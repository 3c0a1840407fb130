"""Expert-parallel worker: one process per GPU (spawned by test_gpu_ep.py).

Each rank holds its shard of a synthetic layer (experts [base, base+per) of
the same seeded arena), exchanges the IPC handles of its exchange window
through a gloo group on 127.0.0.1, and runs smoe_cuda_moe_layer_ep. Rank 0
checks y against the CPU oracle for the whole layer; every rank checks the
routing. Exit code 0 = pass; the failure is printed otherwise.

    python tests/ep_worker.py RANK WORLD PORT FMT [SHAPE]

SHAPE: 30b (d 2048, d_ff 768; default) or 235b (d 4096, d_ff 1536), both
through the layer kernel's in-kernel exchange at batch 1 and 3; or 235b-b32:
batch 32 (BASELINE config 3's batched case) through smoe_cuda_moe_layer_shard
(each rank's experts on the expert-grouped path) and an NCCL reduce of the
ranks' partial sums to rank 0.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "s-moe_b200"), os.path.join(ROOT, "tests")):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle as O  # noqa: E402
import smoe_cuda as S  # noqa: E402

TIGHT = 1e-4   # same bound as the single-GPU fused-layer parity tests


def rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def main():
    rank, world, port, fmt = (int(a) for a in sys.argv[1:5])
    shape = sys.argv[5] if len(sys.argv) > 5 else "30b"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    d, dff, E, k = (2048, 768, 128, 8) if shape == "30b" else (4096, 1536, 128, 8)
    if shape == "235b-b32":
        sys.exit(grouped_main(rank, world, fmt, d, dff, E, k))
    arena, stride, off = O.make_experts(fmt, E, d, dff, 41)
    router = O.normal_bf16(41, 6, E * d, 0.0, 0.02)
    base, per = S.ep_partition(E, world, rank)
    ctx = S.Context(rank)
    d_shard = torch.from_numpy(np.ascontiguousarray(arena[base:base + per])).cuda()
    d_router = torch.from_numpy(router.view(np.int16)).cuda()
    vault = S.make_layer(d_shard, stride, off, per, d, dff, fmt, d_router)
    tstride = S.tiled_stride(fmt, d, dff)
    tbuf = torch.empty(per * tstride, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()                 # the shard was copied on torch's stream
    shard = ctx.prepack_layer(vault, tbuf, tstride)
    ctx.synchronize()

    handles = S.ep_exchange_handles(ctx.ep_export(), world)
    ctx.ep_attach(rank, world, handles)
    dist.barrier()                           # every rank attached before any launch

    failures = []
    for call in range(3 if shape == "30b" else 2):
        for B in (1, 3):
            xb = O.normal_bf16(200 + call, 5 + B, B * d)
            x = torch.from_numpy(xb.view(np.int16)).cuda() if rank == 0 else None
            y = torch.zeros(B, d, dtype=torch.float32, device="cuda") if rank == 0 else None
            ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
            w = torch.zeros(B, k, dtype=torch.float32, device="cuda")
            ctx.moe_layer_ep(shard, E, base, x, S.DTYPE_BF16, B, k, True, y, S.DTYPE_F32, ids, w)
            ctx.synchronize()
            gid = ids.cpu().numpy().view(np.uint32)
            for t in range(B):
                xt = O.bf16_to_f32(xb[t * d:(t + 1) * d])
                ref, rids, rw = O.moe_layer(fmt, xt, router, arena, stride, E, d, dff, k)
                if not (gid[t] == rids).all():
                    failures.append(f"rank {rank} call {call} B {B} tok {t}: ids {gid[t]} != {rids}")
                if rank == 0:
                    e = rel_err(y.cpu().numpy()[t], ref)
                    if e >= TIGHT:
                        failures.append(f"call {call} B {B} tok {t}: rel_err {e:.3e}")
    dist.barrier()
    ctx.close()
    dist.destroy_process_group()
    if failures:
        print("\n".join(failures))
        sys.exit(1)
    print(f"rank {rank}: ok")


def grouped_main(rank, world, fmt, d, dff, E, k, B=32):
    """Batch 32: every rank routes the same x over the whole router, runs
    its experts' slots (vault layout, expert-grouped path), and the partial
    sums meet on rank 0 through an NCCL reduce."""
    import datetime
    nccl = dist.new_group(backend="nccl", timeout=datetime.timedelta(seconds=120))
    arena, stride, off = O.make_experts(fmt, E, d, dff, 43)
    router = O.normal_bf16(43, 6, E * d, 0.0, 0.02)
    base, per = S.ep_partition(E, world, rank)
    ctx = S.Context(rank)
    stream = torch.cuda.Stream()              # a real stream: handle 0 would select the context's own
    ctx.set_stream(stream.cuda_stream)
    d_shard = torch.from_numpy(np.ascontiguousarray(arena[base:base + per])).cuda()
    d_router = torch.from_numpy(router.view(np.int16)).cuda()
    shard = S.make_layer(d_shard, stride, off, per, d, dff, fmt, d_router)
    failures = []
    for call in range(2):
        xb = O.normal_bf16(300 + call, 5, B * d)
        x = torch.from_numpy(xb.view(np.int16)).cuda()
        y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
        ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):          # the reduce is ordered after the shard's kernels
            ctx.moe_layer_shard(shard, E, base, x, S.DTYPE_BF16, B, k, True, y, ids)
            dist.reduce(y, dst=0, group=nccl)    # the NCCL combine
        torch.cuda.synchronize()
        gid = ids.cpu().numpy().view(np.uint32)
        for t in range(0, B, 4):
            xt = O.bf16_to_f32(xb[t * d:(t + 1) * d])
            ref, rids, _ = O.moe_layer(fmt, xt, router, arena, stride, E, d, dff, k)
            if not (gid[t] == rids).all():
                failures.append(f"rank {rank} call {call} tok {t}: ids {gid[t]} != {rids}")
            if rank == 0:
                e = rel_err(y.cpu().numpy()[t], ref)
                if e >= TIGHT:
                    failures.append(f"call {call} tok {t}: rel_err {e:.3e}")
    dist.barrier()
    ctx.close()
    dist.destroy_process_group()
    if failures:
        print("\n".join(failures))
        return 1
    print(f"rank {rank}: ok (batch {B}, grouped + NCCL reduce)")
    return 0


if __name__ == "__main__":
    main()
