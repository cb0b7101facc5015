"""Thread-per-rank stand-in for torch.distributed on one GPU (test helper).

``emulated_group(W)`` patches the collectives the engines call
(all_to_all_single, all_gather_into_tensor, all_reduce) with in-process
copies between W threads, each acting as one rank on the same device, so
multi-rank host logic runs with the real kernels on a single GPU.  The
kernels never wait on each other (each rank's launches are independent),
and the copies are ordered by the device's default stream.
"""
import threading
from concurrent.futures import ThreadPoolExecutor
from contextlib import contextmanager

import torch
import torch.distributed as dist

DEV = torch.device("cuda", 0)


@contextmanager
def emulated_group(world):
    """torch.distributed replaced by an in-process thread-per-rank transport."""
    local = threading.local()
    barrier = threading.Barrier(world, timeout=120)
    slots = [None] * world
    names = ("is_initialized", "get_world_size", "get_rank", "all_to_all_single", "all_gather_into_tensor",
             "get_backend")
    saved = {n: getattr(dist, n) for n in names}

    def all_to_all(output, input, group=None):
        slots[local.rank] = input.clone()
        barrier.wait()
        output.copy_(torch.stack([slots[s][local.rank] for s in range(world)]))
        barrier.wait()

    def all_gather(output, input, group=None):
        slots[local.rank] = input.clone()
        barrier.wait()
        output.copy_(torch.cat(slots).view(output.shape))
        barrier.wait()

    dist.is_initialized = lambda: True
    dist.get_world_size = lambda group=None: world
    dist.get_rank = lambda group=None: local.rank
    dist.all_to_all_single = all_to_all
    dist.all_gather_into_tensor = all_gather
    dist.get_backend = lambda group=None: "emulated"  # not "nccl": the engines keep the collective exchange

    def run(fn):
        def worker(rank):
            local.rank = rank
            torch.cuda.set_device(DEV)
            try:
                return fn(rank)
            except BaseException:
                barrier.abort()
                raise
        with ThreadPoolExecutor(max_workers=world) as ex:
            return list(ex.map(worker, range(world)))
    try:
        yield run
    finally:
        for n, f in saved.items():
            setattr(dist, n, f)


