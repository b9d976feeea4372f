"""Row-block sharding of one exact product across GPUs (one process per GPU).

C's row block r depends only on A's row block r and all of B, so rank r owns
rows [r0, r1) of A and C.  The exchange steps are the only collectives:

1. B is all-gathered from the row blocks each rank holds (raw entries: for
   the 64-bit configuration that is 8 bytes per entry, the smallest form B
   takes anywhere on the path -- its int8 digit planes are 16 B/entry and the
   transformed F stack 120 B/entry), then every rank packs and transforms B
   locally;
2. C's rows reach rank 0 in the plane-major [RL][n][n] layout of the
   reference: by default each rank's final kernel stores them straight into
   rank 0's buffer through a CUDA IPC mapping (PeerOutput); or with grouped
   point-to-point NCCL transfers plane by plane (gather_planes_to_root).

The helpers work on any torch.distributed backend (NCCL on GPUs, gloo on
CPU tensors in the tests).
"""
from __future__ import annotations


def row_range(n: int, world: int, rank: int, align: int = 128):
    """Balanced split of n rows into world blocks, boundaries on `align`
    multiples where possible (whole tcgen05 row tiles per rank)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad world/rank")
    units = (n + align - 1) // align
    lo = units * rank // world
    hi = units * (rank + 1) // world
    return min(n, lo * align), min(n, hi * align)


def all_ranges(n: int, world: int, align: int = 128):
    return [row_range(n, world, r, align) for r in range(world)]


def _bytes(t):
    import torch
    return t.contiguous().view(-1).view(torch.uint8)


def allgather_rows(local, full, n_cols: int, ranges, group=None):
    """Gather row blocks (row-major, n_cols elements per row) of every rank
    into `full` on every rank.  Data moves as raw bytes (any element type;
    16-bit limbs included).  Unequal blocks are handled with one broadcast
    per rank from its own slice."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    row = n_cols * full.element_size()
    fb = full.view(-1).view(__import__("torch").uint8)
    lb = _bytes(local)
    sizes = {(r1 - r0) for r0, r1 in ranges}
    r0, r1 = ranges[rank]
    if len(sizes) == 1:
        dist.all_gather_into_tensor(fb, lb, group=group)
        return full
    fb[r0 * row:r1 * row].copy_(lb)
    for src in range(world):
        a, b = ranges[src]
        if b > a:
            dist.broadcast(fb[a * row:b * row], src=src, group=group)
    return full


def gather_planes_to_root(local, full, n: int, RL: int, ranges, group=None, root: int = 0):
    """local: [RL][rows_r][n] output rows of this rank (flat).  On the root,
    full: [RL][n][n] (flat) receives every rank's rows plane by plane."""
    import torch
    import torch.distributed as dist
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    r0, r1 = ranges[rank]
    rows = r1 - r0
    es = local.element_size()
    lv = local.view(-1).view(torch.uint8).view(RL, rows, n * es) if rows else None
    ops = []
    if rank == root:
        fv = full.view(-1).view(torch.uint8).view(RL, n, n * es)
        if rows:
            fv[:, r0:r1, :].copy_(lv)
        for src in range(world):
            a, b = ranges[src]
            if src == root or b <= a:
                continue
            for w in range(RL):
                ops.append(dist.P2POp(dist.irecv, fv[w, a:b, :], src, group=group))
    elif rows:
        for w in range(RL):
            ops.append(dist.P2POp(dist.isend, lv[w].contiguous() if not lv[w].is_contiguous()
                                  else lv[w], root, group=group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return full


class _DeviceArray:
    """__cuda_array_interface__ of a raw device buffer (for torch.as_tensor)."""

    def __init__(self, ptr, count, typestr):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


class PeerOutput:
    """A device buffer owned by rank `root` and mapped into every other rank
    of the node with CUDA IPC.  Each rank's final kernel (inverse + carry)
    stores its rows of C straight into it over NVLink -- the compute and the
    gather of C are one step, with no separate collective.  `ptr` is this
    rank's device address of the buffer; on the root, `tensor` views it.

    Construction and close() are collective.  If the root cannot allocate or
    any rank cannot map the buffer, every rank undoes what it set up and
    raises, so no rank is left waiting in a later collective.  `lib` is the
    loaded library (tests pass a stand-in)."""

    _TYPESTR = {"uint16": "<u2", "float32": "<f4", "float64": "<f8"}
    _ESIZE = {"uint16": 2, "float32": 4, "float64": 8}

    def __init__(self, count: int, dtype: str, group=None, root: int = 0, lib=None):
        import ctypes as C

        import torch.distributed as dist

        if lib is None:
            from ._lib import lib
        self._lib = lib
        self.group, self.root = group, root
        self.rank = dist.get_rank(group)
        self.count, self.dtype = count, dtype
        self.esize = self._ESIZE[dtype]
        self._tensor = None
        ptr = C.c_void_p()
        handle = (C.c_char * 64)()
        payload = [None]
        ok, err = True, ""
        if self.rank == root:
            rc = lib.mfftgpu_ipc_alloc(count * self.esize, C.byref(ptr), handle)
            if rc:
                ok, err = False, f"mfftgpu_ipc_alloc failed ({rc})"
            else:
                payload = [bytes(handle)]
        dist.broadcast_object_list(payload, src=root, group=group)
        if self.rank != root:
            if payload[0] is None:
                ok, err = False, "the root rank could not allocate the shared output"
            else:
                buf = (C.c_char * 64).from_buffer_copy(payload[0])
                rc = lib.mfftgpu_ipc_open(buf, C.byref(ptr))
                if rc:
                    ok, err = False, f"mfftgpu_ipc_open failed ({rc})"
        self.ptr = ptr.value if ok else None
        oks = [None] * dist.get_world_size(group)
        dist.all_gather_object(oks, ok, group=group)
        if not all(oks):
            self._release()
            raise RuntimeError(err or "the shared output could not be mapped on another rank")

    @property
    def tensor(self):
        """The whole buffer as a flat tensor on the root (None elsewhere)."""
        if self.rank != self.root or self.ptr is None:
            return None
        if self._tensor is None:
            import torch
            self._tensor = torch.as_tensor(
                _DeviceArray(self.ptr, self.count, self._TYPESTR[self.dtype]), device="cuda")
        return self._tensor

    def _release(self):
        # mappings are closed on every rank before the root frees the memory
        import torch.distributed as dist
        self._tensor = None
        dist.barrier(group=self.group)
        if self.rank != self.root and self.ptr is not None:
            self._lib.mfftgpu_ipc_close(self.ptr)
        dist.barrier(group=self.group)
        if self.rank == self.root and self.ptr is not None:
            self._lib.mfftgpu_ipc_free(self.ptr)
        self.ptr = None

    def close(self):
        if getattr(self, "_closed", False):
            return
        self._closed = True
        self._release()


def sub_ranges(r0: int, r1: int, nsub: int, align: int = 256):
    """Split [r0, r1) into nsub pieces on `align` boundaries (fewer if short)."""
    rows = r1 - r0
    units = (rows + align - 1) // align
    nsub = max(1, min(nsub, units))
    cuts = [r0 + min(rows, (units * k // nsub) * align) for k in range(nsub + 1)]
    return [(cuts[k], cuts[k + 1]) for k in range(nsub) if cuts[k + 1] > cuts[k]]


def plan_subblocks(ranges, nsub: int, align: int = 256):
    """Per rank, exactly the same number of sub-blocks (the smallest count
    any rank can make, at least 1); each rank's last sub-block runs to the
    end of its rows, and a rank without rows gets empty (r1, r1) blocks.
    Returns subs[rank][k] = (a, b)."""
    per = [sub_ranges(a, b, nsub, align) if b > a else [] for a, b in ranges]
    k = max(1, min((len(x) for x in per if x), default=1))
    out = []
    for (a, b), x in zip(ranges, per):
        if not x:
            out.append([(b, b)] * k)
            continue
        x = x[:k]
        x[-1] = (x[-1][0], b)
        out.append(x)
    return out


def gather_sub_to_root_async(local, full, n: int, RL: int, seg_of_rank, group=None, root: int = 0):
    """Post (without waiting) the transfers of one sub-block index: every
    rank's rows seg_of_rank[r] = (a, b) go plane by plane into full
    [RL][n][n] on the root; local is this rank's [RL][b-a][n] block.
    Returns the list of work handles to wait on."""
    import torch
    import torch.distributed as dist
    rank = dist.get_rank(group)
    a0, b0 = seg_of_rank[rank]
    es = local.element_size()
    ops = []
    if rank == root:
        fv = full.view(-1).view(torch.uint8).view(RL, n, n * es)
        if b0 > a0:
            fv[:, a0:b0, :].copy_(local.view(-1).view(torch.uint8).view(RL, b0 - a0, n * es))
        for src, (a, b) in enumerate(seg_of_rank):
            if src == root or b <= a:
                continue
            for w in range(RL):
                ops.append(dist.P2POp(dist.irecv, fv[w, a:b, :], src, group=group))
    elif b0 > a0:
        lv = local.view(-1).view(torch.uint8).view(RL, b0 - a0, n * es)
        for w in range(RL):
            ops.append(dist.P2POp(dist.isend, lv[w], root, group=group))
    return dist.batch_isend_irecv(ops) if ops else []
