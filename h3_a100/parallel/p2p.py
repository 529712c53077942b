"""Peer-memory transport: collectives done by this package's own kernels over NVLink.

``PeerComm`` has the ``TorchComm`` interface, but the data-moving collectives
of the training step run in hand-written kernels (``csrc/comm/p2p.cu``) that
read and write the other GPUs' memory directly:

* frozen-weight shards live in symmetric buffers, so gathering a unit needs
  no synchronisation at all (the shards never change): by default one
  copy-engine memcpy per peer shard, which leaves every SM to the compute it
  overlaps, or a pull kernel;
* the AdaLN projection is computed on each rank's rows and the results are
  stored straight into every rank's output buffer (GEMV + all-gather fused);
* each LoRA optimizer step is ONE cooperative kernel: reduce-scatter of the
  fp32 gradients, global-norm exchange, clip + AdamW on this rank's shard of
  the optimizer state, and an all-gather of the new bf16 parameters by
  stores into every replica (``FlatAdamW`` routes here).  With
  ``H3_P2P_MULTIMEM=1`` (and NVLink SHARP in the fabric) the reduce-scatter
  is an in-switch ``multimem.ld_reduce`` and the all-gather a ``multimem.st``
  through the buffers' multicast addresses, so each byte crosses this GPU's
  links once.

Symmetric buffers come from ``torch.distributed._symmetric_memory`` (equal
allocations mapped into every peer); cross-GPU ordering uses epoch flags in
one symmetric int32 buffer, with bounded waits in the kernels.  Scalars and
object gathers (logging, the census) stay on NCCL through the base class.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .comm import TorchComm, _Pending

SIGNAL_INTS = 64          # [4 slots x 8 senders] flags + 8 float slots
# fused LoRA step scratch: 16 scalar slots ([15] = global gradient norm) + one
# partial sum of squares per block of the cooperative grid (at most 8 per SM)
LORA_SCRATCH_FLOATS = 16 + 8 * 160
SLOT_ADALN = 3


class PeerComm(TorchComm):
    name = "p2p"

    def __init__(self, group=None, device: torch.device | None = None, *, kernels=None) -> None:
        super().__init__(group, device)
        if not self.cuda:
            raise ValueError("PeerComm needs CUDA devices")
        if self.world_size > 8:
            raise ValueError("PeerComm supports up to 8 ranks (one NVLink domain)")
        import torch.distributed._symmetric_memory as symm_mem

        self._symm = symm_mem
        self.group = group or dist.group.WORLD
        self.kernels = kernels
        from .. import _C

        self.C = _C
        self._handles: dict[int, tuple[object, int]] = {}
        self.flags = self.alloc_symmetric(SIGNAL_INTS, torch.int32)
        self.epoch = 0
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.limit_ns = int(30e9)
        self.bar = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.scratch = torch.zeros(LORA_SCRATCH_FLOATS, dtype=torch.float32, device=self.device)
        self.bytes_peer = 0
        # In-switch reduction (multimem) is opt-in: at 2 and 4 ranks the
        # unicast peer loads measured faster (1.15 vs 1.87 ms and 1.44 vs
        # 1.74 ms for a 198 M-parameter LoRA step).  H3_P2P_MULTIMEM=1 enables it.
        self.use_multimem = os.environ.get("H3_P2P_MULTIMEM", "0") == "1"
        # Frozen-weight gathers run on the copy engines by default (one
        # cudaMemcpyAsync per shard, no SM time): measured at 2 GPUs, a
        # 226.5 MB gather overlapping the QKV GEMM slowed it by 1.9 % on the
        # copy engines and by 9.6 % as the pull kernel (0.25 vs 0.21 ms for the
        # gather alone, hidden behind the previous block either way).
        # H3_P2P_GATHER=kernel selects the pull kernel.
        self.gather_engine = os.environ.get("H3_P2P_GATHER", "copy")
        if self.gather_engine not in ("kernel", "copy"):
            raise ValueError(f"H3_P2P_GATHER must be kernel or copy, not {self.gather_engine!r}")

    # ---------------------------------------------------------------- buffers
    def alloc_symmetric(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """Zero-filled tensor whose storage is mapped into every peer (collective call)."""
        t = self._symm.empty(int(numel), dtype=dtype, device=self.device)
        t.zero_()
        handle = self._symm.rendezvous(t, self.group.group_name)
        self._handles[t.data_ptr()] = (handle, 0)
        dist.barrier(group=self.group, device_ids=[self.device.index])
        return t

    def alloc_shard(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        return self.alloc_symmetric(numel, dtype)

    def multicast_ptr(self, t: torch.Tensor) -> int:
        """NVLS multicast address of ``t`` (0 when unavailable or disabled).

        A load through it returns the sum over every rank's copy (reduced in
        the NVSwitch); a store through it lands in every rank's copy.  Used
        only with ``H3_P2P_MULTIMEM=1`` and when the fabric has multicast
        support.
        """
        if not self.use_multimem:
            return 0
        base = t.untyped_storage().data_ptr()
        entry = self._handles.get(base)
        if entry is None:
            raise KeyError("tensor is not a symmetric buffer of this communicator")
        mc = int(getattr(entry[0], "multicast_ptr", 0) or 0)
        return mc + (t.data_ptr() - base) if mc else 0

    def peer_ptrs(self, t: torch.Tensor) -> list[int]:
        base = t.untyped_storage().data_ptr()
        entry = self._handles.get(base)
        if entry is None:
            raise KeyError("tensor is not a symmetric buffer of this communicator")
        handle, _ = entry
        offset = t.data_ptr() - base
        return [int(p) + offset for p in handle.buffer_ptrs]

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def check_status(self) -> None:
        code = int(self.status[0].item())
        if code:
            self.status.zero_()
            raise RuntimeError(f"peer-memory collective failed with status {code}")

    # ---------------------------------------------------------------- frozen-weight gather
    def all_gather_async(self, shard: torch.Tensor, total: int) -> _Pending:
        if self.world_size == 1:
            return super().all_gather_async(shard, total)
        self._stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self._stream):
            out = self._buffer(total, shard.dtype)
            t0 = self.timeline.event(self._stream) if self.timeline is not None else None
            gather = self.C.p2p_all_gather_ce if self.gather_engine == "copy" else self.C.p2p_all_gather
            gather(self.peer_ptrs(shard), shard.numel() * shard.element_size(), out)
            if t0 is not None:
                label = "all_gather_copy_engines" if self.gather_engine == "copy" else "all_gather_pull"
                self.timeline.add("comm", label, t0, self.timeline.event(self._stream))
            event = torch.cuda.Event()
            event.record(self._stream)
        self.bytes_gathered += out.numel() * out.element_size()
        self.bytes_peer += (self.world_size - 1) * shard.numel() * shard.element_size()
        return _Pending(out, event)

    # ---------------------------------------------------------------- all-gather fused into a GEMM
    def gather_spec(self, shard: torch.Tensor, rows_per_rank: int, flags: torch.Tensor):
        """Arguments for ``NativeKernels.linear_allgather``: every rank's shard
        of a row-sharded weight (symmetric buffer of ``rows_per_rank`` rows)
        and this rank's int32 per-N-tile counters (reset by each call).  No
        barrier is needed: the shards are written once."""
        return self.peer_ptrs(shard), int(rows_per_rank), flags

    # ---------------------------------------------------------------- AdaLN GEMV + all-gather
    def adaln_project(self, temb: torch.Tensor, w_rows: torch.Tensor, b_rows: torch.Tensor,
                      out: torch.Tensor) -> torch.Tensor:
        """out (symmetric, [R, world*rows] fp32) <- every rank's rows of SiLU(temb) W^T + b."""
        self.C.adaln_project_gather(temb.to(torch.bfloat16).contiguous(), w_rows, b_rows, self.peer_ptrs(out),
                                    self.peer_ptrs(self.flags), self.rank, self.next_epoch(), SLOT_ADALN,
                                    self.status, self.limit_ns)
        return out

    # ---------------------------------------------------------------- fused LoRA optimizer step
    def lora_step(self, opt, lr: float) -> None:
        store = opt.store
        b1, b2 = opt.betas
        self.C.lora_rs_adamw(self.peer_ptrs(store.grad), self.peer_ptrs(store.flat), self.peer_ptrs(self.flags),
                             self.rank, self.next_epoch(), opt.master, opt.exp_avg, opt.exp_avg_sq, self.scratch,
                             self.bar, lr, b1, b2, opt.eps, opt.weight_decay, opt.step_count, opt.max_grad_norm,
                             self.status, self.limit_ns, self.multicast_ptr(store.grad),
                             self.multicast_ptr(store.flat))
