"""Data parallelism over camera views: one process per GPU, replicated Gaussians, one all-reduce per step.

    views = shard_views(cameras, rank, world)          # round-robin, 8 / world views each for config C4
    grads = FlatGradients(n, rest_bases, device)       # six gradient tensors as views of ONE buffer
    ... backward of each view with out=grads.views (accumulate=True for the second view onwards) ...
    grads.all_reduce()                                 # one NCCL all-reduce (sum) of 59 floats per Gaussian
    ... the same fused Adam step on every rank ...

The reference has no multi-GPU path (every job is single-GPU); this is the sharding the benchmark spec asks
for: independent views plus one exchange step. PeerAdam below fuses that exchange with the optimizer: one kernel
per rank reads its slice of every rank's gradients over NVLink, applies Adam, and writes the slice of parameters
back to every rank (plain peer loads and stores; no multicast loads), or does the same through NVLink multicast.
CompactPeerAdam sends each view's SH gradients as six floats per Gaussian (colour gradient and view direction) and
forms the products on the owner; NcclAdam is the reduce-scatter / all-gather baseline. make_exchange picks one.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

GROUPS = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")


def widths(rest_bases: int = 15) -> tuple[int, ...]:
    return (3, 3, 4, 1, 3, 3 * rest_bases)


def shard_views(views: list, rank: int, world: int) -> list:
    """Round-robin share of the batch's views for this rank (every rank gets >= 1 when len(views) >= world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return [views[k] for k in range(rank, len(views), world)]


class FlatGradients:
    """The per-Gaussian gradients of all six parameter groups in one contiguous float32 buffer, so that a
    step needs exactly one collective."""

    def __init__(self, n: int, rest_bases: int = 15, device=None):
        self.n = n
        self.rest_bases = rest_bases
        self.flat = torch.zeros(sum(widths(rest_bases)) * n, dtype=torch.float32, device=device)
        shapes = ((n, 3), (n, 3), (n, 4), (n, 1), (n, 1, 3), (n, rest_bases, 3))
        self.views, off = [], 0
        for w, shp in zip(widths(rest_bases), shapes):
            self.views.append(self.flat[off:off + w * n].view(shp))
            off += w * n

    def zero_(self) -> None:
        self.flat.zero_()

    def add_(self, grads) -> None:
        for v, g in zip(self.views, grads):
            v.add_(g.reshape(v.shape))

    def all_reduce(self, group=None) -> None:
        """Sum over ranks (no-op without an initialised process group of more than one rank)."""
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)


# ---------------------------------------------------------------------------------------------
# Fused data-parallel Adam over peer memory (csrc/dp_adam.cu)
# ---------------------------------------------------------------------------------------------

def owned_slice(total: int, rank: int, world: int) -> tuple[int, int]:
    """The elements [lo, hi) of a flat vector of `total` elements that rank `rank` of `world` updates: equal
    chunks rounded up to a multiple of 4 elements (16-byte aligned starts), the last ones possibly short or empty."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    chunk = ((total + world - 1) // world + 3) // 4 * 4
    lo = min(rank * chunk, total)
    return lo, min(lo + chunk, total)


class _CudaArray:
    """A device address range exposed through the CUDA array interface, so torch can view it without a copy."""

    def __init__(self, ptr: int, numel: int):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<f4", "data": (ptr, False), "version": 2}


class PeerFlat:
    """A flat float32 vector in device memory that every rank of the group can address: this rank's buffer
    as a tensor, and the device addresses of every rank's buffer as this GPU sees them (its own and peer
    mappings opened from the handles the ranks exchange)."""

    def __init__(self, numel: int, group=None, device=None):
        from . import _lib as L

        self._L = L
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.numel = numel
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        L.call("splat_peer_alloc", max(4 * numel, 16), ctypes.byref(ptr), handle)
        self._own = ptr.value
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs, self._opened = [], []
        for k, h in enumerate(handles):
            if k == self.rank:
                self.ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            L.call("splat_peer_open", (ctypes.c_ubyte * 64).from_buffer_copy(h), ctypes.byref(p))
            self.ptrs.append(p.value)
            self._opened.append(p.value)
        self.tensor = torch.as_tensor(_CudaArray(self._own, numel), device=device)

    def close(self) -> None:
        """Unmap the peers' buffers, wait for every rank to do the same, then free this rank's buffer."""
        if self._own is None:
            return
        self.tensor = None
        for p in self._opened:
            self._L.call("splat_peer_close", p)
        self._opened = []
        dist.barrier(group=self.group)
        self._L.call("splat_peer_free", self._own)
        self._own = None


class MulticastFlat:
    """A flat float32 vector allocated as PyTorch symmetric memory: this rank's buffer as a tensor, every rank's
    buffer address (`ptrs`) and the NVLink multicast address bound to all of them (`mc`, 0 when the node has no
    NVLS). Made in two steps: the constructor allocates this rank's buffer (local, no collective); bind() is the
    collective rendezvous that exchanges the addresses, which every rank must enter."""

    def __init__(self, numel: int, group=None, device=None):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.numel = numel
        self.tensor = symm_mem.empty(max(numel, 4), dtype=torch.float32, device=device)
        self.tensor.zero_()
        self._handle = None
        self.ptrs: list = []
        self.mc = 0

    def bind(self) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self._handle = symm_mem.rendezvous(self.tensor, self.group if self.group is not None else dist.group.WORLD)
        self.ptrs = list(self._handle.buffer_ptrs)
        self.mc = int(self._handle.multicast_ptr)

    def close(self, barrier: bool = True) -> None:
        if self.tensor is None:
            return
        if barrier:
            dist.barrier(group=self.group)  # nobody addresses this buffer any more
        self.tensor = None
        self._handle = None


_SETUP_ERRORS = (RuntimeError, ImportError, AttributeError, OSError)


def _all_ranks(flag: int, group, device) -> bool:
    ok = torch.tensor([int(flag)], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    return bool(int(ok.item()))


def agree_on_buffers(make, count: int, group=None, device=None):
    """Make `count` multicast buffers on every rank and return them where every rank has them all with a multicast
    address; otherwise close this rank's (no rank has addressed them, so without a barrier) and return None. Every
    rank gets the same answer, also when the buffers fail on some ranks only.

    Two agreement points keep the ranks' collectives in step: `make()` allocates one buffer locally (no
    collective), and the ranks agree that every allocation succeeded before any of them enters the buffers'
    collective `bind()` (the rendezvous), in the same order on every rank; they agree again on the multicast
    addresses. A rank whose allocation fails therefore never leaves the others waiting inside a rendezvous."""
    made = []
    try:
        for _ in range(count):
            made.append(make())
        allocated = 1
    except _SETUP_ERRORS:
        allocated = 0
    if _all_ranks(allocated, group, device):
        try:
            for b in made:
                b.bind()
            usable = int(all(b.mc != 0 for b in made))
        except _SETUP_ERRORS:
            usable = 0
        if _all_ranks(usable, group, device):
            return made
    for b in made:
        b.close(barrier=False)
    return None


class _BackwardInto:
    """The autograd hook of gs3d._Rasterize (the one FusedAdam(fuse_backward=True) uses), for the exchanges that take
    six gradient tensors: while the exchange is open, the backward of a diff_rasterize call on its six parameter
    tensors writes its gradients into `grads` (a step's first view stores, later views add) instead of returning
    them, and step() finds them in place with nothing to copy."""

    def _hook_backward(self) -> None:
        from . import gs3d

        self._written = 0
        gs3d._Rasterize.fused_optimizer = self

    def _unhook_backward(self) -> None:
        from . import gs3d

        if gs3d._Rasterize.fused_optimizer is self:
            gs3d._Rasterize.fused_optimizer = None

    def _owns(self, six) -> bool:
        return len(self.params) == 6 and all(t.data_ptr() == p.data_ptr() and t.shape == p.shape
                                             for t, p in zip(six, self.params))

    def _defer(self, pending, six) -> None:
        pending.preprocess(out=self.grads, accumulate=self._written > 0)
        self._written += 1

    def _take_grads(self, grads) -> None:
        """step()'s `grads` (e.g. the leaves' .grad): added to what the hooked backward wrote this step, or copied
        into the buffer when it wrote nothing; None entries are skipped."""
        if grads is not None:
            for v, g in zip(self.grads, grads):
                if g is None:
                    continue
                if self._written:
                    v.add_(g.reshape(v.shape))
                else:
                    v.copy_(g.reshape(v.shape))
        self._written = 0


class PeerAdam(_BackwardInto):
    """Data-parallel Adam for replicated parameters, one fused kernel per step instead of an all-reduce of the
    gradients followed by the same Adam step on every rank.

    Parameters and gradients live in peer-addressable flat buffers (`params`, `grads`: per-group views). Each rank
    updates the slice `owned_slice(total, rank, world)` of the flat vector: its kernel sums that slice's gradients
    over the ranks (peer loads), applies Adam with the slice's moments, and writes the updated slice into every
    rank's parameters (peer stores). Two stream-ordered barriers (one-element all-reduces) bracket the kernel.
    Bias corrections and the per-element update are those of FusedAdam; the gradient sum is taken in rank order.

    nvls: use NVLink SHARP when the node has it (the buffers come from PyTorch's symmetric memory, the kernel sums
    through multimem.ld_reduce and writes through multimem.st). Per rank and direction its links then carry
    (G + 1) / G slices-worth of the vector against 2 (G - 1) / G for peer loads and stores: more at G = 2 (1.5 vs
    1), fewer from G = 4 on (1.25 vs 1.5; 1.125 vs 1.75 at G = 8). Measured on the 3M-Gaussian C3 state (the kernel
    alone, maximum over the ranks): at G = 2 1.86 ms multicast against 1.07 ms peer; at G = 4 1.69 ms multicast
    against 1.66 ms peer. Without an explicit `nvls`, the form exchange_for() picks for the rank count is taken.
    """

    def __init__(self, tensors, lrs, group=None, betas=(0.9, 0.999), eps: float = 1e-15, nvls: bool | None = None):
        from . import _lib as L

        self._L = L
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise RuntimeError("PeerAdam supports at most 8 ranks")
        dev = tensors[0].device
        self.shapes = [tuple(t.shape) for t in tensors]
        sizes = [t.numel() for t in tensors]
        self.total = sum(sizes)
        if nvls is None:
            nvls = exchange_for(self.world) == "nvls"  # the six-tensor forms' choice
        self.nvls = False
        if nvls and self.world > 1:
            padded = (self.total + 3) // 4 * 4  # the multicast kernel moves whole 16-byte groups
            bufs = agree_on_buffers(lambda: MulticastFlat(padded, group, dev), 2, group, dev)
            if bufs is not None:
                self.param_buf, self.grad_buf, self.nvls = bufs[0], bufs[1], True
        if not self.nvls:
            self.param_buf = PeerFlat(self.total, group, dev)
            self.grad_buf = PeerFlat(self.total, group, dev)
        self.params, self.grads, self.segments, off = [], [], [], 0
        for t, n, lr in zip(tensors, sizes, lrs):
            pv = self.param_buf.tensor[off:off + n].view(t.shape)
            pv.copy_(t.detach())
            self.params.append(pv)
            self.grads.append(self.grad_buf.tensor[off:off + n].view(t.shape))
            self.segments.append((off, off + n, float(lr)))
            off += n
        self.lo, self.hi = owned_slice(self.param_buf.numel if self.nvls else self.total, self.rank, self.world)
        self.exp_avg = torch.zeros(max(self.hi - self.lo, 1), dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros_like(self.exp_avg)
        self.betas, self.eps, self.t = betas, eps, 0
        self._tiny = torch.zeros(1, dtype=torch.float32, device=dev)
        self._seg = (_Segment * len(self.segments))(*[_Segment(a, b, lr) for a, b, lr in self.segments])
        self._gptr = (ctypes.c_void_p * 8)(*self.grad_buf.ptrs)
        self._pptr = (ctypes.c_void_p * 8)(*self.param_buf.ptrs)
        self._hook_backward()
        dist.barrier(group=group)  # every rank's initial parameters are in place

    def _barrier(self) -> None:
        dist.all_reduce(self._tiny, group=self.group)

    @torch.no_grad()
    def step(self, grads=None) -> None:
        """One step. `grads` (a list of per-group tensors, e.g. the leaves' .grad) is first copied into this rank's
        gradient buffer (added, when a hooked diff_rasterize backward already wrote it); leave it None when the
        backward wrote into `grads` directly."""
        self._take_grads(grads)
        self.t += 1
        stream = torch.cuda.current_stream(self.exp_avg.device).cuda_stream
        self._barrier()
        ev = _kernel_events(self)
        if self.nvls:
            self._L.call("adam_step_dp_nvls", self.lo, self.hi, self.grad_buf.mc, self.param_buf.mc,
                         self._L.ptr(self.param_buf.tensor), self._L.ptr(self.exp_avg), self._L.ptr(self.exp_avg_sq),
                         len(self.segments), ctypes.addressof(self._seg), self.t, float(self.betas[0]),
                         float(self.betas[1]), float(self.eps), stream)
        else:
            self._L.call("adam_step_dp_fused", self.world, self.rank, ctypes.addressof(self._gptr),
                         ctypes.addressof(self._pptr), self.lo, self.hi, self._L.ptr(self.exp_avg),
                         self._L.ptr(self.exp_avg_sq), len(self.segments), ctypes.addressof(self._seg), self.t,
                         float(self.betas[0]), float(self.betas[1]), float(self.eps), stream)
        if ev:
            ev[1].record()
        self._barrier()

    def close(self) -> None:
        self._unhook_backward()
        torch.cuda.synchronize()
        self.params = self.grads = []
        self.param_buf.close()
        self.grad_buf.close()


def _kernel_events(ex):
    """When ex.kernel_events is a list (a caller timing the exchange kernel apart from the barriers around it): a
    pair of CUDA events, the first recorded now on the current stream, appended to it; else None."""
    if not isinstance(getattr(ex, "kernel_events", None), list):
        return None
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    ex.kernel_events.append((a, b))
    return a, b


class NcclAdam(_BackwardInto):
    """PeerAdam's step through NCCL collectives, for comparison and for nodes without peer access: a reduce-scatter
    of the flat gradient vector (rank r receives the summed slice it owns), Adam on that slice with the slice's
    moments (the exchange kernels' segmented Adam on one rank: adam_step_dp_fused with G = 1), and an all-gather
    of the updated parameter slices into every rank's flat parameter vector. The same interface as PeerAdam
    (`params`, `grads` as per-group views of flat buffers, step(), close()); the vector is padded to G equal
    slices of a multiple of 4 elements. Gradient sums follow NCCL's reduction order (at G = 2 one addition, the
    same bits as PeerAdam)."""

    def __init__(self, tensors, lrs, group=None, betas=(0.9, 0.999), eps: float = 1e-15):
        from . import _lib as L

        self._L = L
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        dev = tensors[0].device
        self.shapes = [tuple(t.shape) for t in tensors]
        sizes = [t.numel() for t in tensors]
        self.total = sum(sizes)
        self.chunk = ((self.total + self.world - 1) // self.world + 3) // 4 * 4
        padded = self.chunk * self.world
        self.param_flat = torch.zeros(padded, dtype=torch.float32, device=dev)
        self.grad_flat = torch.zeros(padded, dtype=torch.float32, device=dev)
        self.params, self.grads, self.segments, off = [], [], [], 0
        for t, n, lr in zip(tensors, sizes, lrs):
            pv = self.param_flat[off:off + n].view(t.shape)
            pv.copy_(t.detach())
            self.params.append(pv)
            self.grads.append(self.grad_flat[off:off + n].view(t.shape))
            self.segments.append((off, off + n, float(lr)))
            off += n
        self.lo = self.rank * self.chunk
        self.hi = min(self.lo + self.chunk, self.total) if self.lo < self.total else self.lo
        self.grad_slice = torch.zeros(self.chunk, dtype=torch.float32, device=dev)
        self.exp_avg = torch.zeros(self.chunk, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros_like(self.exp_avg)
        self.betas, self.eps, self.t = betas, eps, 0
        self._seg = (_Segment * len(self.segments))(*[_Segment(a, b, lr) for a, b, lr in self.segments])
        # The kernel reads gradient element e (lo <= e < hi) at grads[0] + e: the slice's base, moved back by lo.
        self._gptr = (ctypes.c_void_p * 8)(self.grad_slice.data_ptr() - 4 * self.lo)
        self._pptr = (ctypes.c_void_p * 8)(self.param_flat.data_ptr())
        self._hook_backward()
        dist.barrier(group=group)

    @torch.no_grad()
    def step(self, grads=None) -> None:
        self._take_grads(grads)
        self.t += 1
        ev = _kernel_events(self)
        dist.reduce_scatter_tensor(self.grad_slice, self.grad_flat, op=dist.ReduceOp.SUM, group=self.group)
        stream = torch.cuda.current_stream(self.exp_avg.device).cuda_stream
        self._L.call("adam_step_dp_fused", 1, 0, ctypes.addressof(self._gptr), ctypes.addressof(self._pptr), self.lo,
                     self.hi, self._L.ptr(self.exp_avg), self._L.ptr(self.exp_avg_sq), len(self.segments),
                     ctypes.addressof(self._seg), self.t, float(self.betas[0]), float(self.betas[1]), float(self.eps),
                     stream)
        mine = self.param_flat[self.rank * self.chunk:(self.rank + 1) * self.chunk]
        dist.all_gather_into_tensor(self.param_flat, mine, group=self.group)
        if ev:
            ev[1].record()

    def close(self) -> None:
        self._unhook_backward()
        torch.cuda.synchronize()
        self.params = self.grads = []


def owned_gaussians(n: int, rank: int, world: int) -> tuple[int, int]:
    """The Gaussians [lo, hi) of n whose parameters rank `rank` of `world` updates in the compact exchange: equal
    chunks rounded up to a multiple of 4 Gaussians, the last ones possibly short or empty."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    chunk = ((n + world - 1) // world + 3) // 4 * 4
    lo = min(rank * chunk, n)
    return lo, min(lo + chunk, n)


def compact_layout(n: int, rest_bases: int, views: int) -> dict:
    """Element offsets of the compact exchange's flat buffers for n Gaussians (adam_step_dp_compact): the parameter
    vector (means, scales, rotations, opacities, sh0, sh_rest) and the gradient vector (the four non-SH groups,
    then one block of six-float records per view)."""
    p_off, off = {}, 0
    for name, w in zip(GROUPS, widths(rest_bases)):
        p_off[name] = (off, off + w * n)
        off += w * n
    g_off = {name: p_off[name] for name in GROUPS[:4]}
    rec = [(11 * n + 6 * n * v, 11 * n + 6 * n * (v + 1)) for v in range(views)]
    return {"params": p_off, "param_total": off, "grads": g_off, "records": rec, "grad_total": (11 + 6 * views) * n}


class CompactPeerAdam:
    """PeerAdam with compact SH gradients (adam_step_dp_compact). A view's SH gradients are the products
    basis_k(view direction) x colour gradient, so each rank stores per view and Gaussian six floats (the colour
    gradient and the direction: gs3d.PendingBackward.preprocess_records) in place of its 3 (rest_bases + 1) SH
    gradients; the owner of a Gaussian forms every rank's products with the preprocess backward's rounding and
    sums them (views in view order, ranks in rank order). The non-SH groups are summed as in PeerAdam. Per step a
    rank's links carry (11 + 6 views) floats per Gaussian of gradients instead of 59, and the full parameter
    vector. Rank r owns whole Gaussians (owned_gaussians) and updates all of their parameters.

    `params`: the six parameter tensors as views of the peer-addressable parameter buffer; `grads`: the four
    non-SH gradient tensors; `records[v]`: view v's record block (6n floats). Every step must write all `views`
    record blocks (the first view stores its gradients, the others accumulate into `grads`): through
    gs3d.backward(..., out=grads, records=records[v], accumulate=v > 0), or through autograd - while this object is
    open, the backward of a diff_rasterize call on its six parameter tensors writes the next record block and the
    non-SH gradients here and leaves the tensors' .grad untouched (the hook FusedAdam's fuse_backward uses)."""

    def __init__(self, tensors, lrs, views: int, active_sh_bases: int, group=None, betas=(0.9, 0.999),
                 eps: float = 1e-15):
        from . import _lib as L

        self._L = L
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise RuntimeError("CompactPeerAdam supports at most 8 ranks")
        if views < 1:
            raise ValueError("views must be >= 1")
        tensors = list(tensors)
        dev = tensors[0].device
        self.n = n = tensors[0].shape[0]
        self.rest = tensors[5].shape[1] if tensors[5].dim() == 3 else 0
        self.views, self.active_sh_bases = int(views), int(active_sh_bases)
        self.shapes = [tuple(t.shape) for t in tensors]
        lay = compact_layout(n, self.rest, self.views)
        self.param_buf = PeerFlat(lay["param_total"], group, dev)
        self.grad_buf = PeerFlat(lay["grad_total"], group, dev)
        self.params, self.grads = [], []
        for name, t in zip(GROUPS, tensors):
            a, b = lay["params"][name]
            pv = self.param_buf.tensor[a:b].view(t.shape)
            pv.copy_(t.detach())
            self.params.append(pv)
            if name in lay["grads"]:
                a, b = lay["grads"][name]
                self.grads.append(self.grad_buf.tensor[a:b].view(t.shape))
        self.records = [self.grad_buf.tensor[a:b] for a, b in lay["records"]]
        self.lo, self.hi = owned_gaussians(n, self.rank, self.world)
        cpad = (self.hi - self.lo + 3) // 4 * 4
        self.exp_avg = torch.zeros(max(sum(widths(self.rest)) * cpad, 1), dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros_like(self.exp_avg)
        self.betas, self.eps, self.t = betas, eps, 0
        self._lr = (ctypes.c_double * 6)(*[float(x) for x in lrs])
        self._tiny = torch.zeros(1, dtype=torch.float32, device=dev)
        self._gptr = (ctypes.c_void_p * 8)(*self.grad_buf.ptrs)
        self._pptr = (ctypes.c_void_p * 8)(*self.param_buf.ptrs)
        self._written = 0  # record blocks written through autograd this step
        from . import gs3d

        gs3d._Rasterize.fused_optimizer = self
        dist.barrier(group=group)

    # ---- the autograd hook of gs3d._Rasterize (the same one FusedAdam(fuse_backward=True) uses) ----
    def _owns(self, six) -> bool:
        return len(self.params) == 6 and all(t.data_ptr() == p.data_ptr() and t.shape == p.shape
                                             for t, p in zip(six, self.params))

    def _defer(self, pending, six) -> None:
        if self._written >= self.views:
            raise RuntimeError(f"more than {self.views} views rendered for one step of the compact exchange")
        pending.preprocess_records(self.grads, self.records[self._written], accumulate=self._written > 0)
        self._written += 1

    def _barrier(self) -> None:
        dist.all_reduce(self._tiny, group=self.group)

    @torch.no_grad()
    def step(self, grads=None) -> None:
        """One step. `grads` (e.g. the leaves' .grad after an autograd backward): None, or per group a tensor to add
        to the gradient of the four non-SH groups; SH gradients other than the records cannot be carried."""
        if grads is not None:
            grads = list(grads)
            if any(g is not None for g in grads[4:]):
                raise RuntimeError("the compact exchange carries SH gradients only as the views' records")
            for v, g in zip(self.grads, grads[:4]):
                if g is not None:
                    v.add_(g.reshape(v.shape))
        if 0 < self._written < self.views:
            raise RuntimeError(f"{self._written} of {self.views} views rendered before the step")
        self._written = 0
        self.t += 1
        stream = torch.cuda.current_stream(self.exp_avg.device).cuda_stream
        self._barrier()
        ev = _kernel_events(self)
        self._L.call("adam_step_dp_compact", self.world, self.rank, ctypes.addressof(self._gptr),
                     ctypes.addressof(self._pptr), self.n, self.lo, self.hi, self.views, self.active_sh_bases,
                     self.rest, self._L.ptr(self.exp_avg), self._L.ptr(self.exp_avg_sq), ctypes.addressof(self._lr),
                     self.t, float(self.betas[0]), float(self.betas[1]), float(self.eps), stream)
        if ev:
            ev[1].record()
        self._barrier()

    def close(self) -> None:
        from . import gs3d

        if gs3d._Rasterize.fused_optimizer is self:
            gs3d._Rasterize.fused_optimizer = None
        torch.cuda.synchronize()
        self.params = self.grads = self.records = []
        self.param_buf.close()
        self.grad_buf.close()


def exchange_for(world: int, form: str = "auto", records: bool = False) -> str:
    """The exchange form a step of `world` ranks uses: "peer" (peer loads and stores, adam_step_dp_fused), "nvls"
    (NVLink multicast, adam_step_dp_nvls), "compact" (peer form with compact SH gradients, CompactPeerAdam) or
    "nccl" (NcclAdam). "auto" picks the form measured fastest at that rank count on 8-GPU B200 nodes: among all
    forms when the caller's backward writes the compact form's records (`records`: AUTO_EXCHANGE), else among the
    forms that take the six gradient tensors (AUTO_EXCHANGE_FULL)."""
    if form != "auto":
        if form not in ("peer", "nvls", "compact", "nccl"):
            raise ValueError(f"unknown exchange form {form!r}")
        return form
    if records:
        return AUTO_EXCHANGE.get(world, "compact" if world >= 4 else "peer")
    return AUTO_EXCHANGE_FULL.get(world, "nvls" if world >= 8 else "peer")


# The fastest form per rank count, exchange kernel alone on the C3 state (3M Gaussians, one view per rank), ms:
#   2 ranks: peer 1.065, compact 1.010 (whole C3 step: peer 677 views/s, compact 660), multicast 1.86
#   4 ranks: peer 1.662, multicast 1.685, compact 1.235, NCCL 2.159
AUTO_EXCHANGE = {2: "peer", 4: "compact", 8: "compact"}
AUTO_EXCHANGE_FULL = {2: "peer", 4: "peer", 8: "nvls"}


def make_exchange(tensors, lrs, form: str = "auto", group=None, betas=(0.9, 0.999), eps: float = 1e-15,
                  views: int = 1, active_sh_bases: int = 16, records: bool = False):
    """PeerAdam (peer or multicast form), CompactPeerAdam or NcclAdam for the replicated parameter tensors, by
    exchange_for(world, form, records). views / active_sh_bases: the compact form's views per rank and step, and SH
    bases; records: the caller's backward can write the compact form's records (so "auto" may choose it)."""
    kind = exchange_for(dist.get_world_size(group), form, records)
    if kind == "compact":
        return CompactPeerAdam(tensors, lrs, views, active_sh_bases, group=group, betas=betas, eps=eps)
    if kind == "nccl":
        return NcclAdam(tensors, lrs, group=group, betas=betas, eps=eps)
    return PeerAdam(tensors, lrs, group=group, betas=betas, eps=eps, nvls=(kind == "nvls"))


class _Segment(ctypes.Structure):
    """Mirror of dp_adam_segment in include/splat_b200.h."""

    _fields_ = [("begin", ctypes.c_longlong), ("end", ctypes.c_longlong), ("lr", ctypes.c_double)]
