"""Column-parallel (N-sharded) fp8imma GEMM across the GPUs of one node.

One process per GPU (torch.distributed, NCCL over NVLink/NVSwitch). Rank r
holds weight rows B[r*N/g:(r+1)*N/g, :] (i.e. output columns) and their
scales; activations are replicated. Each rank runs the local sm_100a kernel
into its slice of the full output, then one all-gather assembles D. Because
the reference output layout is col-major ([N, M] row-major), every rank's
slice is one contiguous block, so the gather needs no re-layout.

The reference has no multi-GPU code; this is the BASELINE-mandated N-sharding.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ext


def shard_bounds(N: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, near-equal split of N columns; sizes differ by at most 1
    granule of 16 columns (the kernels' column-tile friendly unit)."""
    if N % world == 0:
        per = N // world
        return rank * per, (rank + 1) * per
    gran = 16
    units = (N + gran - 1) // gran
    base, extra = divmod(units, world)
    start_u = rank * base + min(rank, extra)
    end_u = start_u + base + (1 if rank < extra else 0)
    return min(N, start_u * gran), min(N, end_u * gran)


class ColumnParallelFP8Gemm:
    """Holds this rank's weight shard; __call__(A) returns the full D [N, M]
    (col-major MxN) on every rank."""

    def __init__(self, B_local: torch.Tensor, scales_local: torch.Tensor, N_total: int,
                 group=None, col_scales_f32: torch.Tensor | None = None, local_fn=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.B = B_local.contiguous()
        self.scales = scales_local.contiguous()
        self.col_scales_f32 = None if col_scales_f32 is None else col_scales_f32.contiguous()
        self.N = N_total
        self.n_local = self.B.shape[0]
        if self.world > 1 and N_total % self.world != 0:
            raise ValueError("N_total must divide evenly across ranks for the gather")
        # local_fn(A, B, scales, col_scales_f32, global_scale, a_inv_scale, act_quant, out) -> D [n_local, M];
        # the default is the sm_100a kernel through the torch extension
        self._local_fn = local_fn
        self._ext = None if local_fn is not None else ext()

    def local(self, A: torch.Tensor, out: torch.Tensor | None = None, global_scale: float = 1.0,
              a_inv_scale: float = 1.0, act_quant: str = "tensor") -> torch.Tensor:
        if self._local_fn is not None:
            return self._local_fn(A, self.B, self.scales, self.col_scales_f32, global_scale, a_inv_scale, act_quant,
                                  out)
        D, _ = self._ext.imma_fp8_gemm(A, self.B, self.scales, self.col_scales_f32, global_scale, a_inv_scale,
                                       act_quant, "e4m3", "int8", "float16", "col", False, out)
        return D

    def __call__(self, A: torch.Tensor, global_scale: float = 1.0, a_inv_scale: float = 1.0,
                 act_quant: str = "tensor", out_full: torch.Tensor | None = None) -> torch.Tensor:
        M = A.shape[0]
        if out_full is None:
            out_full = torch.empty(self.N, M, dtype=torch.float16, device=A.device)
        if self.world == 1:
            return self.local(A, out_full, global_scale, a_inv_scale, act_quant)
        mine = out_full.narrow(0, self.rank * self.n_local, self.n_local)
        self.local(A, mine, global_scale, a_inv_scale, act_quant)
        if dist.get_backend(self.group) == "nccl":
            # in place: this rank's slice already sits at its offset of out_full
            dist.all_gather_into_tensor(out_full, mine, group=self.group)
        else:
            parts = list(out_full.chunk(self.world, dim=0))
            dist.all_gather(parts, mine.clone(), group=self.group)
        return out_full


class FusedGatherFP8Gemm:
    """Column-parallel GEMM whose output gather is fused into the kernel
    (fp8imma_gemm_allgather): each rank's epilogue writes its output rows into
    every rank's full output over NVLink, then a flag barrier. The full
    outputs and the signal pad live in torch symmetric memory; two output
    buffers alternate so a call never overwrites what a peer may still read.
    Returns the full col-major D [N_total, M] (a view of the current buffer).
    Small M only (the split-K kernel), int8-exact path, per-tensor scales.
    """

    def __init__(self, B_local: torch.Tensor, scales_local: torch.Tensor, M: int, group=None):
        import ctypes

        import torch.distributed._symmetric_memory as symm_mem

        from . import FP8ImmaGemmArgs, lib

        self._ctypes, self._Args, self._lib = ctypes, FP8ImmaGemmArgs, lib()
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self.B = B_local.contiguous()
        self.scales = scales_local.contiguous()
        self.n_local = self.B.shape[0]
        self.M = M
        dev = self.B.device
        name = self.group.group_name
        try:
            symm_mem.enable_symm_mem_for_group(name)
        except Exception:
            pass
        self.bufs, self.handles = [], []
        for _ in range(2):
            t = symm_mem.empty(self.n_local * self.world, M, dtype=torch.float16, device=dev)
            self.bufs.append(t)
            self.handles.append(symm_mem.rendezvous(t, name))
        self.pad = symm_mem.empty(64, dtype=torch.int32, device=dev)
        self.pad.zero_()
        pad_h = symm_mem.rendezvous(self.pad, name)
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        P = ctypes.c_void_p * self.world
        self._outs = [P(*[ctypes.c_void_p(x) for x in h.buffer_ptrs]) for h in self.handles]
        self._pads = P(*[ctypes.c_void_p(x) for x in pad_h.buffer_ptrs])
        self.epoch = 0

    def __call__(self, A: torch.Tensor, global_scale: float = 1.0, a_inv_scale: float = 1.0,
                 B: torch.Tensor | None = None) -> torch.Tensor:
        """B optionally replaces the stored weight shard for this call (same shape)."""
        assert A.shape[0] == self.M and A.is_contiguous()
        Bw = self.B if B is None else B
        assert Bw.shape == self.B.shape and Bw.is_contiguous()
        self.epoch += 1
        which = self.epoch & 1  # host-side alternation; the barrier epoch itself is counted on the device
        a = self._Args()
        a.path, a.a_type, a.b_format, a.act_quant = 0, {torch.float16: 0, torch.bfloat16: 1, torch.int8: 2}[A.dtype], 0, 0
        a.out_type, a.out_layout = 0, 0
        a.M, a.N, a.K = self.M, self.n_local, A.shape[1]
        a.A, a.B, a.col_scales_u16 = A.data_ptr(), Bw.data_ptr(), self.scales.data_ptr()
        a.global_scale, a.a_inv_scale = float(global_scale), float(a_inv_scale)
        stream = self._ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        err = self._lib.fp8imma_gemm_allgather(self._ctypes.byref(a), self._outs[which], self._pads, self.world,
                                               self.rank, 0, stream)
        if err != 0:
            raise RuntimeError("fp8imma_gemm_allgather failed, cudaError_t=%d" % err)
        return self.bufs[which]
