"""PyTorch operators over the fused kernels, for tensor-parallel linear layers.

    torch.ops.vmm_agg.all_gather_gemm(A_r, B_r, handle)      -> C_r [M, N_r]
    torch.ops.vmm_agg.gemm_reduce_scatter(X_r, W_r, handle)  -> Y_r [M/P, N]

are registered custom operators (torch.library), so they appear as single nodes
to autograd-free inference graphs, torch.compile and the profiler.  `handle`
names an AllGatherGemm / GemmReduceScatter object (its multicast slab and launch
counter), registered with `register()`; the op's fake implementation gives the
output shape without running anything.

ColumnParallelLinear / RowParallelLinear are the two halves of a
tensor-parallel MLP built on them (forward only):

    up   = ColumnParallelLinear(W_up_r)      # x_r [M/P, K]  -> AllGather(x) W_up_r^T  [M, N/P]
    down = RowParallelLinear(W_down_r)       # h_r [M, K/P]  -> rows r of sum_s h_s W_s^T  [M/P, N]
"""
from __future__ import annotations

import itertools

import torch

from . import agg

_OPS: dict[int, object] = {}
_IDS = itertools.count(1)


def register(op) -> int:
    """Makes an AllGatherGemm or GemmReduceScatter callable through torch.ops; returns its handle."""
    h = next(_IDS)
    _OPS[h] = op
    return h


def unregister(handle: int) -> None:
    _OPS.pop(handle, None)


def _op(handle: int):
    try:
        return _OPS[handle]
    except KeyError:
        raise agg.AggError(f"no operator registered under handle {handle}") from None


@torch.library.custom_op("vmm_agg::all_gather_gemm", mutates_args=())
def all_gather_gemm(A_r: torch.Tensor, B_r: torch.Tensor, handle: int) -> torch.Tensor:
    """C_r = AllGather(A_r) . B_r^T through the AllGatherGemm registered as `handle`."""
    return _op(handle)(A_r, B_r)


@all_gather_gemm.register_fake
def _(A_r, B_r, handle):
    op = _op(handle)
    return A_r.new_empty((op.M, B_r.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op("vmm_agg::gemm_reduce_scatter", mutates_args=())
def gemm_reduce_scatter(X_r: torch.Tensor, W_r: torch.Tensor, handle: int) -> torch.Tensor:
    """Y_r = rows r of sum_s X_s . W_s^T through the GemmReduceScatter registered as `handle`."""
    return _op(handle)(X_r, W_r)


@gemm_reduce_scatter.register_fake
def _(X_r, W_r, handle):
    op = _op(handle)
    return X_r.new_empty((op.m_local, W_r.shape[0]), dtype=torch.bfloat16)


class ColumnParallelLinear(torch.nn.Module):
    """y = AllGather(x_r) . W_r^T with the weight shard W_r [N/P, K] of this rank
    (bf16): the up / gate projection of a tensor-parallel MLP, one fused kernel."""

    def __init__(self, weight_r: torch.Tensor, m_local: int, *, group=None, host_group=None, producer: str = "sm"):
        super().__init__()
        self.weight = torch.nn.Parameter(weight_r.contiguous(), requires_grad=False)
        self.op = agg.AllGatherGemm(m_local, weight_r.shape[1], group=group, host_group=host_group,
                                    device=weight_r.device, producer=producer)
        self.handle = register(self.op)

    def forward(self, x_r: torch.Tensor) -> torch.Tensor:
        return torch.ops.vmm_agg.all_gather_gemm(x_r, self.weight, self.handle)

    def close(self):
        unregister(self.handle)
        self.op.close()


class RowParallelLinear(torch.nn.Module):
    """y_r = rows r of sum_s x_s . W_s^T with the weight slice W_r [N, K/P] of this
    rank (bf16): the down projection of a tensor-parallel MLP, one fused kernel."""

    def __init__(self, weight_r: torch.Tensor, m: int, *, group=None, host_group=None):
        super().__init__()
        self.weight = torch.nn.Parameter(weight_r.contiguous(), requires_grad=False)
        self.op = agg.GemmReduceScatter(m, weight_r.shape[0], weight_r.shape[1], group=group,
                                        host_group=host_group, device=weight_r.device)
        self.handle = register(self.op)

    def forward(self, x_r: torch.Tensor) -> torch.Tensor:
        return torch.ops.vmm_agg.gemm_reduce_scatter(x_r, self.weight, self.handle)

    def close(self):
        unregister(self.handle)
        self.op.close()
