"""The combine fused with the cross-rank all-reduce, over NVLink peer memory.

``PeerAllReduce`` is one rank's member of a TP / EP group: every rank owns a
receive area that all ranks write by plain P2P stores (CUDA IPC handles,
exchanged once through ``torch.distributed``). ``finalize`` takes the place of
the reference's ``AllReduceMHC.finalize`` (``all_reduce_mhc.py:1484``) for the
MoE output: rank r's partial is y_r = bf16(bf16(sum_k w rows_r[perm]) + shared_r)
(``all_reduce_mhc.py:528-640``) and the result is bf16 of the fp32 sum of
y_0, ..., y_{n-1} in rank order (the reduce at ``all_reduce_mhc.py:955-977``).
``moe_finalize_all_reduce_rms_norm`` adds the decoder hop's residual + RMSNorm
epilogue (``qwen3_5/sm103/hop/__init__.py:431``) in the same launch.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import check, lib
from .moe import _ptr, _stream


class PeerAllReduce:
    """One rank of a group exchanging MoE outputs through peer memory.

    Collective at construction (every rank of ``group`` must build one with the
    same ``max_tokens`` and ``hidden``); afterwards every ``finalize`` is one
    launch per rank, and all ranks must call it in the same order with the
    same token count. Without an initialized process group it is a group of
    one (the combine alone, through the same kernel)."""

    def __init__(self, max_tokens: int, hidden: int, group=None, device: Optional[torch.device] = None,
                 eps: float = 1e-6):
        import torch.distributed as dist

        grouped = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if grouped else 0
        self.world = dist.get_world_size(group) if grouped else 1
        self.max_tokens, self.hidden, self.eps = int(max_tokens), int(hidden), float(eps)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        h = ctypes.c_void_p()
        check(lib().mm_comm_create(self.rank, self.world, self.max_tokens, self.hidden,
                                   self.device.index, ctypes.byref(h)), "mm_comm_create")
        self.handle = h.value
        try:
            mine = (ctypes.c_ubyte * _lib.MM_IPC_HANDLE_BYTES)()
            check(lib().mm_comm_handle(self.handle, mine), "mm_comm_handle")
            handles = [bytes(mine)]
            if grouped:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(mine), group=group)
            blob = b"".join(handles)
            if len(blob) != self.world * _lib.MM_IPC_HANDLE_BYTES:
                raise RuntimeError("PeerAllReduce: malformed IPC handles from the group")
            table = (ctypes.c_ubyte * len(blob)).from_buffer_copy(blob)
            check(lib().mm_comm_open(self.handle, table), "mm_comm_open")
            if grouped:
                dist.barrier(group=group)
        except BaseException:
            lib().mm_comm_destroy(self.handle)
            self.handle = None
            raise

    @classmethod
    def local_group(cls, max_tokens: int, hidden: int, devices, eps: float = 1e-6) -> list:
        """Every member of a group driven by this one process: rank q on
        ``devices[q]`` (devices may repeat). Each member reaches the others'
        buffers directly (peer access between distinct devices), with no IPC
        and no process group. Returns the members in rank order."""
        world = len(devices)
        members = []
        try:
            for q, dev in enumerate(devices):
                m = cls.__new__(cls)
                m.rank, m.world = q, world
                m.max_tokens, m.hidden, m.eps = int(max_tokens), int(hidden), float(eps)
                m.device = torch.device(dev)
                m.handle = None
                h = ctypes.c_void_p()
                check(lib().mm_comm_create(q, world, m.max_tokens, m.hidden, m.device.index, ctypes.byref(h)),
                      "mm_comm_create")
                m.handle = h.value
                members.append(m)
            table = (ctypes.c_void_p * world)(*(m.handle for m in members))
            for m in members:
                check(lib().mm_comm_open_local(m.handle, table), "mm_comm_open_local")
        except BaseException:
            for m in members:
                m.close()
            raise
        return members

    def set_wait_budget(self, microseconds: int) -> None:
        """Budget of this rank's mailbox polls (default 1.5 s); a poll that runs
        out ends the launch and makes ``check`` raise DeviceTimeoutError."""
        check(lib().mm_comm_set_wait_budget(self.handle, int(microseconds)), "mm_comm_set_wait_budget")

    def _check(self, rows, weights, permuted, shared_output):
        if self.handle is None:
            raise RuntimeError("PeerAllReduce is closed")
        tokens, top_k = weights.shape
        if rows.dtype != torch.bfloat16 or rows.dim() != 2 or rows.shape[1] != self.hidden:
            raise ValueError(f"rows must be bf16 [rows, {self.hidden}]")
        if weights.dtype != torch.float32 or permuted.dtype != torch.int32 or tuple(permuted.shape) != (tokens, top_k):
            raise ValueError("weights fp32 [T, k] and permuted int32 [T, k] expected")
        if shared_output is not None and (shared_output.dtype != torch.bfloat16
                                          or tuple(shared_output.shape) != (tokens, self.hidden)):
            raise ValueError("shared_output must be bf16 [T, H]")
        for t in (rows, weights, permuted, shared_output):
            if t is not None and not t.is_contiguous():
                raise ValueError("finalize inputs must be contiguous")
        return tokens, top_k

    def finalize(self, rows: torch.Tensor, weights: torch.Tensor, permuted: torch.Tensor,
                 shared_output: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """bf16 [T, H]: the group's sum of every rank's finalized partial."""
        tokens, top_k = self._check(rows, weights, permuted, shared_output)
        if out is None:
            out = torch.empty((tokens, self.hidden), dtype=torch.bfloat16, device=rows.device)
        check(lib().mm_finalize_allreduce(self.handle, rows.data_ptr(), weights.data_ptr(), permuted.data_ptr(),
                                          _ptr(shared_output), out.data_ptr(), tokens, top_k, self.hidden,
                                          _stream(rows.device)), "mm_finalize_allreduce")
        return out

    def moe_finalize_all_reduce_rms_norm(self, *, routed_output: torch.Tensor, expert_weights: torch.Tensor,
                                         permuted_indices: torch.Tensor, gated_shared_output: Optional[torch.Tensor],
                                         residual: torch.Tensor, gamma: Optional[torch.Tensor],
                                         norm_out: Optional[torch.Tensor] = None,
                                         residual_out: Optional[torch.Tensor] = None):
        """(norm_out, residual_out), the decoder hop after the MoE
        (qwen3_5/sm103/hop/__init__.py:431): residual_out = bf16(group sum +
        residual), norm_out = RMSNorm(residual_out) * gamma (None without gamma)."""
        tokens, top_k = self._check(routed_output, expert_weights, permuted_indices, gated_shared_output)
        if residual.dtype != torch.bfloat16 or tuple(residual.shape) != (tokens, self.hidden) \
                or not residual.is_contiguous():
            raise ValueError("residual must be contiguous bf16 [T, H]")
        if gamma is not None and (gamma.dtype != torch.bfloat16 or tuple(gamma.shape) != (self.hidden,)):
            raise ValueError("gamma must be bf16 [H]")
        dev = routed_output.device
        if residual_out is None:
            residual_out = torch.empty((tokens, self.hidden), dtype=torch.bfloat16, device=dev)
        if norm_out is None and gamma is not None:
            norm_out = torch.empty((tokens, self.hidden), dtype=torch.bfloat16, device=dev)
        check(lib().mm_finalize_allreduce_norm(
            self.handle, routed_output.data_ptr(), expert_weights.data_ptr(), permuted_indices.data_ptr(),
            _ptr(gated_shared_output), residual.data_ptr(), _ptr(gamma), self.eps, residual_out.data_ptr(),
            _ptr(norm_out) if gamma is not None else None, tokens, top_k, self.hidden, _stream(dev)),
            "mm_finalize_allreduce_norm")
        return (norm_out if gamma is not None else None), residual_out

    def check(self) -> None:
        """Synchronize and raise if a peer never signalled within the device's wait budget."""
        check(lib().mm_comm_check(self.handle), "mm_comm_check")

    def close(self) -> None:
        """Free this rank's buffers (after every rank has finished its last finalize)."""
        if self.handle is not None:
            lib().mm_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
