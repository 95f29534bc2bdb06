"""One rank of the bounded-wait check (test infrastructure; run on two GPUs
under torch.distributed.run by tests/test_tp.py). Both ranks connect and
take one exchange together; then rank 0 alone starts a second exchange with
a short wait limit while rank 1 never publishes (it waits on the host, with
nothing of its own in flight). Rank 0's kernel must give up after the limit,
the host must see NMX_ERR_TIMEOUT, and the context must still run work
afterwards."""
import argparse
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    import torch
    import torch.distributed as dist
    from novamlx_b200 import nmx

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", init_method="env://")
    torch.cuda.set_device(rank)
    ctx = nmx.Context(rank)
    comm = nmx.tp_comm(ctx, rank, world, 64 * 512 * 2, nmx.torch_exchange(dist))
    dev = f"cuda:{rank}"
    part = torch.ones((64, 512), device=dev, dtype=torch.float16)
    res = torch.zeros_like(part)
    out = torch.empty_like(part)
    comm.allreduce_resid(part, res, out)
    ctx.synchronize()
    together = bool(torch.all(out == world).item())
    dist.barrier()
    result = {"rank": rank, "together": together}
    if rank == 0:
        ctx.set_wait_limit(1 << 16)
        t0 = time.perf_counter()
        comm.allreduce_resid(part, res, out)  # no peer publishes this epoch
        try:
            ctx.synchronize()
            result["status"] = "no error"
        except nmx.NmxError as e:
            result["status"] = "timeout" if e.status == nmx.NMX_ERR_TIMEOUT else f"status {e.status}"
            result["message"] = str(e)
        result["seconds"] = time.perf_counter() - t0
        ctx.set_wait_limit(0)
        # the GPU is released and the context still runs work
        x = torch.randn((4, 512), device=dev, dtype=torch.float16)
        y = ctx.rms_norm(x, torch.ones(512, device=dev, dtype=torch.float16))
        ctx.synchronize()
        result["usable_after"] = bool(torch.isfinite(y.float()).all().item())
    dist.barrier()
    comm.close()
    with open(f"{a.out}.rank{rank}.json", "w") as f:
        json.dump(result, f)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
