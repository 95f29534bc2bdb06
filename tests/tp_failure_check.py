"""One rank of the host-side failure check (test infrastructure; run on CPU
under torch.distributed.run with gloo by tests/test_tp.py): rank 1 leaves
before the communicator rendezvous, and rank 0 must learn of it on the host
as an error from the handle exchange, within the process group's short
timeout, instead of waiting for good."""
import datetime
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    import torch.distributed as dist
    from novamlx_b200 import nmx
    rank = int(os.environ["RANK"])
    dist.init_process_group("gloo", init_method="env://", timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        print("rank 1 leaves", flush=True)
        os._exit(0)  # no goodbye: the peer finds out from the transport
    t0 = time.perf_counter()
    try:
        nmx.torch_exchange(dist)(bytes(nmx.IPC_HANDLE_BYTES))
        print("rank 0 not detected", flush=True)
    except Exception as e:  # gloo reports the lost peer or the timeout
        print(f"rank 0 detected after {time.perf_counter() - t0:.1f} s: {type(e).__name__}", flush=True)
    os._exit(0)


if __name__ == "__main__":
    main()
