"""Fused Ulysses exchange of the DiT step over NVLink peer memory.

With P ranks (one GPU each, one node), rank r holds tokens [r*L, (r+1)*L) of
the sequence and attends heads [r*H/P, (r+1)*H/P).  Instead of an
all-to-all after the q/k/v producer and another after the attention, the
kernels store across GPUs themselves:

* ``pasa_dit_qkv_rope_scatter`` writes the normalised, rotated q/k rows and
  the v rows of head h straight into the receive buffer of the rank that
  attends h ([3, H/P, P*L, D] on every rank);
* ``pasa_forward_scatter`` runs PASA on the rank's heads over all tokens and
  writes each output row into the token-major buffer of the rank that owns
  the token ([L, H, D] on every rank), the layout the output projection reads.

The buffers are allocated by the library (``pasa_peer_alloc``) and mapped
into the other processes with CUDA IPC handles, exchanged once with
``all_gather_object``.  A one-element NCCL all-reduce after each scatter,
ordered on the compute stream, is the cross-rank barrier: a rank reads its
buffer only after every rank's scatter kernel has finished, and a scatter
into a buffer starts only after its owner has finished reading the previous
contents (the barrier after the other scatter sits between the two).
"""
from __future__ import annotations

import ctypes
from typing import List

import torch
import torch.distributed as dist

from . import _lib, ops


class _DeviceArray:
    """A library-owned device allocation seen as a torch tensor (zero copy,
    through the CUDA array interface)."""

    def __init__(self, ptr: int, shape, device: torch.device):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}
        with torch.cuda.device(device):
            self.tensor = torch.as_tensor(self, device=device).view(torch.bfloat16)


class UlyssesPeerExchange:
    def __init__(self, group, device: torch.device, heads: int, head_dim: int, tokens_local: int):
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if heads % self.P:
            raise ValueError(f"{heads} heads do not split over {self.P} ranks")
        self.device = device
        self.H, self.D, self.L = heads, head_dim, tokens_local
        self.Hl = heads // self.P
        lib = _lib.load()
        self._lib = lib
        self._local: List[int] = []
        self._opened: List[int] = []

        def alloc(shape):
            nbytes = 2
            for n in shape:
                nbytes *= n
            ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(_lib.PEER_HANDLE_BYTES)
            with torch.cuda.device(device):
                _lib.check("pasa_peer_alloc", lib.pasa_peer_alloc(nbytes, ctypes.byref(ptr),
                                                                  ctypes.cast(handle, ctypes.c_void_p)))
            self._local.append(ptr.value)
            return ptr.value, handle.raw

        qkv_ptr, qkv_h = alloc((3, self.Hl, self.P * self.L, self.D))
        o_ptr, o_h = alloc((self.L, self.H, self.D))
        self.qkv = _DeviceArray(qkv_ptr, (3, self.Hl, self.P * self.L, self.D), device).tensor
        self.obuf = _DeviceArray(o_ptr, (self.L, self.H, self.D), device).tensor
        handles = [None] * self.P
        dist.all_gather_object(handles, (qkv_h, o_h), group=group)
        qkv_ptrs, o_ptrs = [], []
        for r, (hq, ho) in enumerate(handles):
            if r == self.rank:
                qkv_ptrs.append(qkv_ptr)
                o_ptrs.append(o_ptr)
                continue
            for h, out in ((hq, qkv_ptrs), (ho, o_ptrs)):
                ptr = ctypes.c_void_p()
                hbuf = ctypes.create_string_buffer(h, _lib.PEER_HANDLE_BYTES)
                with torch.cuda.device(device):
                    _lib.check("pasa_peer_open", lib.pasa_peer_open(ctypes.cast(hbuf, ctypes.c_void_p),
                                                                    ctypes.byref(ptr)))
                self._opened.append(ptr.value)
                out.append(ptr.value)
        self.qkv_table = torch.tensor(qkv_ptrs, dtype=torch.int64, device=device)
        self.o_table = torch.tensor(o_ptrs, dtype=torch.int64, device=device)
        self._flag = torch.zeros(1, dtype=torch.int32, device=device)

    def barrier(self):
        """Stream-ordered cross-rank barrier (a one-element NCCL all-reduce)."""
        dist.all_reduce(self._flag, group=self.group)

    def scatter_qkv(self, xq, xk, xv, wq, wk, cos, sin, eps: float):
        """q/k RMSNorm + rotary + head scatter of this rank's tokens; returns
        this rank's heads over all tokens as [1, H/P, P*L, D] views (valid
        after the barrier this call ends with)."""
        for t in (xq, xk, xv):
            if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.shape != (1, self.L, self.H * self.D):
                raise ValueError("xq, xk, xv must be contiguous bf16 [1, L, H*D] tensors of this rank's tokens")
        with torch.cuda.device(self.device):
            _lib.check("pasa_dit_qkv_rope_scatter", self._lib.pasa_dit_qkv_rope_scatter(
                ops._stream_ptr(self.device), xq.data_ptr(), xk.data_ptr(), xv.data_ptr(), wq.data_ptr(),
                wk.data_ptr(), cos.data_ptr(), sin.data_ptr(), self.L, self.H, self.D, float(eps),
                self.qkv_table.data_ptr(), self.P, self.rank))
        self.barrier()
        return self.qkv[0][None], self.qkv[1][None], self.qkv[2][None]

    def attention(self, q, k, v, density: float, scale=None):
        """PASA on this rank's heads with each output row stored at its
        token's owner; returns this rank's tokens [1, L, H*D] (valid after the
        barrier this call ends with)."""
        T, D = q.shape[2], q.shape[3]
        scale = D ** -0.5 if scale is None else scale
        NT, NG, NS = _lib.derive(T, density)
        lib = self._lib
        with torch.cuda.device(self.device):
            nbytes = _lib.workspace_size(1, self.Hl, T, D, _lib.BF16, NS)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            _lib.check("pasa_forward_scatter", lib.pasa_forward_scatter(
                ops._stream_ptr(self.device), q.data_ptr(), k.data_ptr(), v.data_ptr(), self.Hl, T, D,
                float(density), float(scale), 1, None, ws.data_ptr(), nbytes, self.o_table.data_ptr(), self.P,
                self.rank * self.Hl, self.H, _lib.ATTN_TCGEN05))
        self.barrier()
        return self.obuf.view(1, self.L, self.H * self.D)

    def close(self):
        """Unmap the peers' buffers and free this rank's (all ranks call it;
        it synchronises so that no rank frees memory another still writes)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.pasa_peer_close(ctypes.c_void_p(p))
            self._opened = []
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._local:
                self._lib.pasa_peer_free(ctypes.c_void_p(p))
            self._local = []
        self.qkv = self.obuf = None
