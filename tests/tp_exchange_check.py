"""One rank of the host-side tensor-parallel rendezvous check (test
infrastructure; run on CPU under torch.distributed.run with gloo by
tests/test_tp.py): every rank contributes a 64-byte handle and must get all
of them back in rank order."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    import torch.distributed as dist
    from novamlx_b200 import nmx
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", init_method="env://")
    got = nmx.torch_exchange(dist)(bytes([rank + 1]) * nmx.IPC_HANDLE_BYTES)
    assert got == [bytes([r + 1]) * nmx.IPC_HANDLE_BYTES for r in range(world)], got
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank} ok", flush=True)


if __name__ == "__main__":
    main()
