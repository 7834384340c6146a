"""Kernel-level entry points (the reference's enqueue-only launch helpers).

Each function enqueues on a CUDA stream (default: torch's current stream) and
returns immediately; tensors are torch CUDA tensors (row-major float32 tiles).
The Workspace owns the checksum vectors, decision records and counters that
the reference keeps in PipelineBuffers (pipeline/buffers.cuh:7-46).
"""
import ctypes

import numpy as np
import torch

from ._lib import CORRECT_INLOOP, call, lib


def _stream(stream):
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def _iptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))


def _dptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def _check_tile(t, rows, cols, name):
    if not (t.is_cuda and t.dtype == torch.float32 and t.dim() == 2 and t.stride(1) == 1):
        raise ValueError(f"{name} must be a row-major float32 CUDA matrix")
    if t.shape[0] < rows or t.shape[1] < cols:
        raise ValueError(f"{name} is {tuple(t.shape)}, need at least ({rows}, {cols})")


class Workspace:
    """Device state of one rank tile (M_b x N_b, K) split into F column fragments."""

    def __init__(self, M_b, N_b, K, counts, offsets, max_iters=0, device_buffer=None):
        self.M_b, self.N_b, self.K = int(M_b), int(N_b), int(K)
        self.counts = np.ascontiguousarray(counts, np.int32)
        self.offsets = np.ascontiguousarray(offsets, np.int32)
        self.F = len(self.counts)
        self.max_iters = int(max_iters)
        self.nbytes = lib.abft_ws_bytes(self.M_b, self.N_b, self.K, self.F, _iptr(self.counts), self.max_iters)
        h = ctypes.c_void_p()
        self._buf = device_buffer
        ptr, nb = ((None, 0) if device_buffer is None else
                   (device_buffer.data_ptr(), device_buffer.numel() * device_buffer.element_size()))
        call("abft_ws_create", self.M_b, self.N_b, self.K, self.F, _iptr(self.counts), _iptr(self.offsets),
             self.max_iters, ptr, nb, ctypes.byref(h))
        self.handle = h

    def close(self):
        if self.handle:
            call("abft_ws_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset_counters(self, stream=None):
        call("abft_ws_reset_counters", self.handle, _stream(stream))

    def counters(self):
        cm = np.zeros(4, np.int32)
        nr = ctypes.c_int()
        call("abft_ws_read_counters", self.handle, _iptr(cm), ctypes.byref(nr))
        return cm, nr.value

    def counters_device_ptr(self):
        return lib.abft_ws_counters_device(self.handle)

    def read_log(self, it_count):
        n = it_count * self.F
        ec = np.zeros(n, np.int32)
        er = np.zeros(n, np.int32)
        rd = np.zeros(n, np.float64)
        call("abft_ws_read_log", self.handle, int(it_count), _iptr(ec), _iptr(er), _dptr(rd))
        return ec.reshape(it_count, self.F), er.reshape(it_count, self.F), rd.reshape(it_count, self.F)

    def read_checksums(self):
        colSumA = np.zeros(self.K, np.float64)
        expRow = np.zeros(self.N_b, np.float64)
        rowSumB = np.zeros(self.F * self.K, np.float64)
        expCol = np.zeros(self.F * self.M_b, np.float64)
        call("abft_ws_read_checksums", self.handle, _dptr(colSumA), _dptr(expRow), _dptr(rowSumB), _dptr(expCol))
        return colSumA, expRow, rowSumB.reshape(self.F, self.K), expCol.reshape(self.F, self.M_b)


def encode(ws, A, B, stream=None):
    """colSumA, expectedRow and the per-fragment localisation checksums."""
    _check_tile(A, ws.M_b, ws.K, "A")
    _check_tile(B, ws.K, ws.N_b, "B")
    call("abft_encode", ws.handle, A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), _stream(stream))


def verify(ws, C, f, tau, injected=False, it=-1, stream=None):
    """Fused actualRow + detect for fragment f of the tile C."""
    _check_tile(C, ws.M_b, ws.N_b, "C")
    call("abft_verify", ws.handle, C.data_ptr(), C.stride(0), int(f), float(tau), int(bool(injected)), int(it),
         _stream(stream))


def calibrate(ws, C, f, out=None, stream=None):
    """|actualRow - expectedRow| of every column of fragment f (float64 CUDA tensor)."""
    _check_tile(C, ws.M_b, ws.N_b, "C")
    if out is None:
        out = torch.empty(int(ws.counts[f]), dtype=torch.float64, device=C.device)
    call("abft_calibrate", ws.handle, C.data_ptr(), C.stride(0), int(f), out.data_ptr(), _stream(stream))
    return out


def localize_correct(ws, C, f, tau, injected=False, golden=None, it=-1, correct_mode=CORRECT_INLOOP, stream=None):
    """Gated localisation and correction of fragment f."""
    _check_tile(C, ws.M_b, ws.N_b, "C")
    gp, ldg = (None, 0) if golden is None else (golden.data_ptr(), golden.stride(0))
    call("abft_localize_correct", ws.handle, C.data_ptr(), C.stride(0), int(f), float(tau), int(bool(injected)),
         gp, ldg, int(it), int(correct_mode), _stream(stream))


def drain(ws, C0, C1, repeats, golden=None, stream=None):
    """Post-loop correction: apply the fixes that localize_correct queued in
    drain mode to the buffers C0 / C1 that still hold their iteration (the last
    two of `repeats`), counting restores against golden when given."""
    gp, ldg = (None, 0) if golden is None else (golden.data_ptr(), golden.stride(0))
    call("abft_drain", ws.handle, C0.data_ptr(), C1.data_ptr(), C0.stride(0), gp, ldg, int(repeats),
         _stream(stream))


def inject_add(C, row, col, delta=1.0e6, stream=None):
    call("abft_inject_add", C.data_ptr(), C.stride(0), int(row), int(col), float(delta), _stream(stream))


def inject_bitflip(C, row, col, bit, stream=None):
    call("abft_inject_bitflip", C.data_ptr(), C.stride(0), int(row), int(col), int(bit), _stream(stream))
