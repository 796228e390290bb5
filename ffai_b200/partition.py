"""Multi-GPU partitioning of segment-batched attention, one process per GPU.

Every (segment, head) is independent, so the work is split by segment with
no collective on the data path: each rank computes its own segments and
copies its output rows into its slice of one host output buffer (the host
gather).  The buffer is a shared-memory file every rank maps, so the slices
land in a single array at precomputed offsets.

There is nothing to partition in the reference (a single process, one
window at a time, text_decoder.rs:1069-1076); this module exists because the
B200 build spreads segment batches over the 8 GPUs of one box.
"""

from __future__ import annotations

import datetime
import heapq
import mmap
import os

import numpy as np


def contiguous_ranges(n_items: int, n_ranks: int):
    """Split range(n_items) into n_ranks contiguous ranges, sizes differing by <= 1."""
    base, extra = divmod(n_items, n_ranks)
    out, start = [], 0
    for r in range(n_ranks):
        size = base + (1 if r < extra else 0)
        out.append((start, start + size))
        start += size
    return out


def lpt_assign(costs, n_ranks: int):
    """Longest-processing-time-first assignment of items with `costs` to ranks.

    Returns (assignment list of item indices per rank, load per rank).  The
    makespan is within 4/3 of optimal (Graham's bound); for ragged segments
    the cost is the attention work, proportional to L^2.
    """
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(n_ranks)]
    heapq.heapify(heap)
    assign = [[] for _ in range(n_ranks)]
    load = [0.0] * n_ranks
    for i in order:
        l, r = heapq.heappop(heap)
        assign[r].append(i)
        load[r] = l + costs[i]
        heapq.heappush(heap, (load[r], r))
    for a in assign:
        a.sort()
    return assign, load


def ragged_assignment(lengths, n_ranks: int):
    """Segments of `lengths` to ranks by LPT on L^2 (attention work).

    Also returns the token load per rank, the balance the workload names."""
    costs = [float(L) * float(L) for L in lengths]
    assign, load = lpt_assign(costs, n_ranks)
    tokens = [int(sum(lengths[i] for i in a)) for a in assign]
    return assign, load, tokens


class SharedHostBuffer:
    """A host buffer shared by all ranks of one node through /dev/shm.

    Each rank maps the same file; rank r writes only its own byte range, so
    no locking is needed.  `pin()` page-locks the mapping for this process's
    CUDA context so device-to-host copies into it run at full PCIe rate.
    """

    def __init__(self, name: str, nbytes: int, create: bool):
        self.path = os.path.join("/dev/shm", name)
        self.nbytes = int(nbytes)
        flags = os.O_RDWR | (os.O_CREAT if create else 0)
        fd = os.open(self.path, flags, 0o600)
        try:
            if create:
                os.ftruncate(fd, self.nbytes)
            self.map = mmap.mmap(fd, self.nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        finally:
            os.close(fd)
        self.array = np.frombuffer(self.map, dtype=np.uint8)
        self._pinned_ptr = None

    def view(self, dtype, shape, offset: int = 0):
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        return self.array[offset:offset + n].view(dtype).reshape(shape)

    def pin(self) -> bool:
        """Register the mapping with CUDA (cudaHostRegister); False if refused."""
        import torch
        ptr = self.array.ctypes.data
        rt = torch.cuda.cudart()
        err = rt.cudaHostRegister(ptr, self.nbytes, 0)
        ok = int(err) == 0 if not isinstance(err, tuple) else int(err[0]) == 0
        if ok:
            self._pinned_ptr = ptr
        return ok

    def close(self, unlink: bool = False):
        if self._pinned_ptr is not None:
            import torch
            torch.cuda.cudart().cudaHostUnregister(self._pinned_ptr)
            self._pinned_ptr = None
        self.array = None
        try:
            self.map.close()
        except BufferError:
            pass
        if unlink:
            try:
                os.unlink(self.path)
            except FileNotFoundError:
                pass


class RankGroup:
    """The ranks of one node, one process per GPU, as a launcher (torchrun)
    describes them in RANK / LOCAL_RANK / WORLD_SIZE / MASTER_*.

    The process group carries only control traffic: barriers, the max over
    ranks of a device time, sums of counters and a gather of small objects
    (checksums).  No tensor of the path crosses it.  `backend` is "nccl" on
    the GPU box (control tensors on the rank's GPU) or "gloo" (CPU tensors),
    which the CPU tests use.
    """

    def __init__(self, backend: str = "nccl", timeout_s: float = 180.0):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.timeout_s = timeout_s
        self.pg = False

    def _device(self):
        import torch
        return torch.device("cuda", self.local) if self.backend == "nccl" else torch.device("cpu")

    def init(self):
        import torch
        if self.backend == "nccl":
            torch.cuda.set_device(self.local)
        if self.world > 1:
            import torch.distributed as dist
            kw = {"device_id": self._device()} if self.backend == "nccl" else {}
            dist.init_process_group(self.backend,
                                    timeout=datetime.timedelta(seconds=self.timeout_s), **kw)
            self.pg = True
        return self

    def barrier(self):
        if self.pg:
            import torch.distributed as dist
            if self.backend == "nccl":
                dist.barrier(device_ids=[self.local])
            else:
                dist.barrier()

    def _reduce(self, x: float, op) -> float:
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=self._device())
        dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch.distributed as dist
        return self._reduce(x, dist.ReduceOp.MAX)

    def sum(self, x: float) -> float:
        if not self.pg:
            return x
        import torch.distributed as dist
        return self._reduce(x, dist.ReduceOp.SUM)

    def gather_objects(self, obj):
        if not self.pg:
            return [obj]
        import torch.distributed as dist
        out = [None] * self.world
        dist.all_gather_object(out, obj)
        return out

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()
            self.pg = False


def open_shared_output(group: RankGroup, name: str, nbytes: int) -> SharedHostBuffer:
    """The node's host output buffer: rank 0 creates it, the others attach
    after a barrier.  Every rank then writes only its own slice."""
    buf = None
    if group.rank == 0:
        buf = SharedHostBuffer(name, nbytes, create=True)
    group.barrier()
    if group.rank != 0:
        buf = SharedHostBuffer(name, nbytes, create=False)
    return buf


def gather_verified(group: RankGroup, local_slice: np.ndarray, whole: np.ndarray | None):
    """Checksum of checksums: every rank reports the checksum of the result it
    computed; rank 0 compares their sum with the checksum of the gathered
    buffer.  Returns True/False on rank 0, None elsewhere."""
    sums = group.gather_objects(checksum(local_slice))
    if group.rank != 0:
        return None
    return checksum(whole) == sum(sums) % 2**64


def checksum(a: np.ndarray) -> int:
    """Order-independent 64-bit checksum of an array's bytes (sum of u64 words)."""
    b = np.ascontiguousarray(a).view(np.uint8)
    pad = (-b.size) % 8
    if pad:
        b = np.concatenate([b, np.zeros(pad, np.uint8)])
    return int(b.view(np.uint64).sum(dtype=np.uint64))
