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
