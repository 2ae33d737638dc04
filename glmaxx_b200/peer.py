"""Peer-mapped buffers of a tensor-parallel group, and the peer form of the finish.

The reference reduces the ranks' FC2 partials with an NCCL all-reduce
(crates/glm-engine/src/manifest.rs:228) and then forms the layer output
(finish_sparse_layer_oracle, crates/glm-reference/src/routed_fc2.rs:214-258).
Here one kernel does both over NVLink: every rank allocates one device block
(glmaxx_device_alloc) with the same layout -- a signal buffer, then the named
buffers -- and sends its CUDA IPC handle to the others over the process group.
Each rank then maps every other rank's block (glmaxx_ipc_open), so the finish can
read every rank's partial and, in the two-shot form, write into every rank's
outputs (glmaxx_moe_finish_peer_launch).

The process group carries only the handles (64 bytes per rank, once) and the
barriers around setup, reset and teardown; no collective runs on the data path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import abi

ALIGN = 256
_TYPESTR = {torch.float32: "<f4", torch.bfloat16: "<i2", torch.int16: "<i2",
            torch.uint8: "|u1", torch.int32: "<i4"}


@dataclass(frozen=True)
class Slot:
    offset: int
    shape: tuple
    dtype: torch.dtype

    @property
    def nbytes(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n * torch.empty((), dtype=self.dtype).element_size()


def plan_layout(buffers: dict, ranks: int) -> tuple[dict, int, int]:
    """Offsets of the signal buffer and of each named buffer (in the order given,
    each 256-byte aligned) inside one rank's block.  Every rank computes the same
    layout from the same arguments.  Returns (slots, signal_bytes, total_bytes)."""
    if not 1 <= ranks <= 8:
        raise ValueError(f"ranks must be 1..8, got {ranks}")
    signal = 256
    off = signal
    slots = {}
    for name, (shape, dtype) in buffers.items():
        if dtype not in _TYPESTR:
            raise ValueError(f"{name}: unsupported dtype {dtype}")
        slot = Slot(off, tuple(int(d) for d in shape), dtype)
        slots[name] = slot
        off += (slot.nbytes + ALIGN - 1) // ALIGN * ALIGN
    return slots, signal, off


class CudaIpc:
    """The C-ABI calls the group needs; a test replaces it with a fake."""

    def __init__(self):
        self.L = abi.load()

    def alloc(self, nbytes: int) -> int:
        p = ctypes.c_uint64()
        abi.check(self.L.glmaxx_device_alloc(nbytes, ctypes.byref(p)), "device_alloc")
        return p.value

    def free(self, ptr: int) -> None:
        abi.check(self.L.glmaxx_device_free(ptr), "device_free")

    def handle(self, ptr: int) -> bytes:
        h = (ctypes.c_uint8 * 64)()
        abi.check(self.L.glmaxx_ipc_handle(ptr, h), "ipc_handle")
        return bytes(h)

    def open(self, handle: bytes) -> int:
        h = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
        p = ctypes.c_uint64()
        abi.check(self.L.glmaxx_ipc_open(h, ctypes.byref(p)), "ipc_open")
        return p.value

    def close(self, ptr: int) -> None:
        abi.check(self.L.glmaxx_ipc_close(ptr), "ipc_close")

    def zero(self, ptr: int, nbytes: int) -> None:
        device_view(ptr, (nbytes // 4,), torch.int32, torch.cuda.current_device()).zero_()
        torch.cuda.current_stream().synchronize()


class _Array:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def device_view(ptr: int, shape, dtype: torch.dtype, device) -> torch.Tensor:
    """A torch tensor over device memory this module owns (no copy)."""
    t = torch.as_tensor(_Array(ptr, shape, _TYPESTR[dtype]), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


class PeerGroup:
    """Buffers that every rank of `group` maps, and the peer finish over them.

    buffers: {name: (shape, dtype)}, the same on every rank.  Collective: every
    rank constructs it (and calls close()) at the same point."""

    def __init__(self, buffers: dict, group=None, device=None, backend=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.ranks = dist.get_world_size(group)
        self.device = device
        self.backend = backend if backend is not None else CudaIpc()
        self.slots, self.signal_bytes, self.total = plan_layout(buffers, self.ranks)
        self.base = self.backend.alloc(self.total)
        handles = [None] * self.ranks
        dist.all_gather_object(handles, self.backend.handle(self.base), group=group)
        self.bases = [self.base if p == self.rank else self.backend.open(handles[p])
                      for p in range(self.ranks)]
        self._views = {}
        self.status = None
        self.reset_signals()

    # ------------------------------------------------------------ addresses
    def pointer(self, name: str, rank: int | None = None) -> int:
        r = self.rank if rank is None else rank
        return self.bases[r] + self.slots[name].offset

    def pointers(self, name: str) -> list[int]:
        return [self.pointer(name, r) for r in range(self.ranks)]

    def signal_pointers(self) -> list[int]:
        return list(self.bases)

    def tensor(self, name: str) -> torch.Tensor:
        """This rank's buffer `name` as a torch tensor."""
        if name not in self._views:
            s = self.slots[name]
            self._views[name] = device_view(self.pointer(name), s.shape, s.dtype, self.device)
        return self._views[name]

    # ------------------------------------------------------------ lifetime
    def reset_signals(self) -> None:
        """Zero this rank's signal buffer, then wait for every rank (after a
        peer timeout, or before the first finish).  Every rank's finish kernels
        have ended before any buffer is zeroed."""
        if self.device is not None or torch.cuda.is_initialized():
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.backend.zero(self.base, self.signal_bytes)
        dist.barrier(group=self.group)

    def close(self) -> None:
        dist.barrier(group=self.group)
        for p, b in enumerate(self.bases):
            if p != self.rank:
                self.backend.close(b)
        dist.barrier(group=self.group)
        self.backend.free(self.base)
        self.bases = []
        self._views = {}

    # ------------------------------------------------------------ the finish
    def finish_descriptors(self, partial: str, residual: torch.Tensor | None = None,
                           attention: torch.Tensor | None = None, out_f32=None, out_bf16=None,
                           norm_bf16=None, hidden: int = 0, eps: float = 1e-6,
                           mode: str = "auto", status: torch.Tensor | None = None,
                           rows: tuple[int, int] | None = None, row_elems: int = 0):
        """(finish descriptor, peer descriptor) for the peer finish of buffer
        `partial`.  Outputs are buffer names of this group (any mode) or local
        tensors (one-shot only).  rows=(lo, hi) with row_elems elements per row
        finishes only those rows of every buffer (a token chunk of the step); a
        local residual or output tensor is then the chunk's own rows."""
        if rows is None:
            first, elements = 0, self.slots[partial].nbytes // 4
        else:
            first, elements = rows[0] * row_elems, (rows[1] - rows[0]) * row_elems
            if elements <= 0 or first + elements > self.slots[partial].nbytes // 4:
                raise ValueError(f"rows {rows} outside the buffer")
        outs = {"f32": out_f32, "bf16": out_bf16, "norm": norm_bf16}
        named = all(v is None or isinstance(v, str) for v in outs.values())
        if mode == "auto":
            mode = "two" if named and two_shot_pays(elements, self.ranks) else "one"
        if mode not in ("one", "two"):
            raise ValueError(f"mode must be 'auto', 'one' or 'two', got {mode!r}")
        if mode == "two" and not named:
            raise ValueError("the two-shot finish writes every rank's outputs: name group buffers")

        def at(name, rank=None):
            # element `first` of a named buffer
            size = torch.empty((), dtype=self.slots[name].dtype).element_size()
            return self.pointer(name, rank) + first * size

        def own(v):
            if v is None:
                return 0
            return at(v) if isinstance(v, str) else v.data_ptr()

        keep = []

        def array(values):
            a = (ctypes.c_uint64 * len(values))(*values)
            keep.append(a)
            return ctypes.addressof(a)

        d = abi.MoeFinishDescriptor.new(
            abi_version=abi.MOE_FINISH_ABI_VERSION, ranks=self.ranks, elements=elements,
            residual_f32=residual.data_ptr() if residual is not None and
            residual.dtype == torch.float32 else 0,
            residual_bf16=residual.data_ptr() if residual is not None and
            residual.dtype == torch.bfloat16 else 0,
            attention_f32=0 if attention is None else attention.data_ptr(),
            partials_f32=array([at(partial, r) for r in range(self.ranks)]),
            output_f32=own(out_f32), output_bf16=own(out_bf16), norm_bf16=own(norm_bf16),
            hidden=hidden, eps=eps)
        p = abi.MoePeerDescriptor.new(
            abi_version=abi.MOE_PEER_ABI_VERSION,
            flags=abi.PEER_TWO_SHOT if mode == "two" else abi.PEER_ONE_SHOT, rank=self.rank,
            signals_u32=array(self.signal_pointers()),
            status_u32=0 if status is None else status.data_ptr())
        if mode == "two":
            every = lambda n: array([at(n, r) for r in range(self.ranks)])
            p.outputs_f32 = every(out_f32) if out_f32 else 0
            p.outputs_bf16 = every(out_bf16) if out_bf16 else 0
            p.norms_bf16 = every(norm_bf16) if norm_bf16 else 0
        d._arrays = keep  # the arrays are read at launch time
        return d, p

    def finish(self, partial: str, **kw) -> None:
        """Peer finish of buffer `partial` on the current stream (every rank calls
        it at the same point of its stream); see finish_descriptors."""
        d, p = self.finish_descriptors(partial, **kw)
        abi.check(abi.load().glmaxx_moe_finish_peer_launch(
            ctypes.byref(d), ctypes.byref(p),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "moe_finish_peer_launch")


def two_shot_pays(elements: int, ranks: int) -> bool:
    """Two-shot moves (N-1)/N of the partial across NVLink each way per rank
    against N-1 partials inbound for one-shot, for one more pass of stores and a
    system-scope fence per CTA.  Measured on two B200s: one-shot wins at 1.5 MB
    (10.7 vs 14.3 us), two-shot from 12.6 MB on (31 vs 35 us); with more ranks the
    one-shot inbound volume grows N-1 times, so two-shot wins from about 1 MB."""
    nbytes = elements * 4
    return nbytes >= (8 << 20) if ranks == 2 else (ranks > 2 and nbytes >= (1 << 20))
