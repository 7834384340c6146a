"""One rank's online ABFT pipeline (pass_baseline / pass_online_loop) over the C ABI."""
import ctypes

import numpy as np
import torch

from . import host
from ._lib import (ADD_FAULT_DELTA, CORRECT_DRAIN, CORRECT_INLOOP, OnlineArgs, OnlineResult, SessionCfg, call,
                   lib)


def _dptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


class OnlineSession:
    """Protected SGEMM C = A @ B on one rank tile with double-buffered C.

    A (M_b x K), B (K x N_b) are row-major float32 CUDA tensors owned by the
    caller; the session allocates the two C buffers (the two OnlineSlots).
    """

    def __init__(self, A, B, frags=None, counts=None, offsets=None, verify_priority=-1, max_iters=256):
        if not (A.is_cuda and B.is_cuda and A.dtype == torch.float32 and B.dtype == torch.float32):
            raise ValueError("A and B must be float32 CUDA tensors")
        self.A, self.B = A.contiguous(), B.contiguous()
        self.M_b, self.K = self.A.shape
        K2, self.N_b = self.B.shape
        if K2 != self.K:
            raise ValueError("inner dimensions differ")
        if counts is None:
            counts, offsets = host.split_dim(self.N_b, int(frags or 1))
        self.counts = np.ascontiguousarray(counts, np.int32)
        self.offsets = np.ascontiguousarray(offsets, np.int32)
        self.F = len(self.counts)
        dev = self.A.device
        # row pitch host.c_pitch(N_b): padded where a dense pitch would slow
        # the verify kernel; C[i] is the M_b x N_b view of each buffer
        ldc = host.c_pitch(self.N_b)
        self.C = [torch.empty((self.M_b, ldc), dtype=torch.float32, device=dev)[:, :self.N_b] for _ in range(2)]
        self.golden = None
        self.max_iters = int(max_iters)
        cfg = SessionCfg()
        cfg.M_b, cfg.N_b, cfg.K, cfg.F = self.M_b, self.N_b, self.K, self.F
        cfg.counts = self.counts.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
        cfg.offsets = self.offsets.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
        cfg.dA, cfg.lda = self.A.data_ptr(), self.A.stride(0)
        cfg.dB, cfg.ldb = self.B.data_ptr(), self.B.stride(0)
        cfg.dC0, cfg.dC1, cfg.ldc = self.C[0].data_ptr(), self.C[1].data_ptr(), self.C[0].stride(0)
        cfg.verify_priority = int(verify_priority)
        cfg.max_iters = self.max_iters
        torch.cuda.synchronize(dev)
        h = ctypes.c_void_p()
        with torch.cuda.device(dev):
            call("abft_session_create", ctypes.byref(cfg), ctypes.byref(h))
        self.handle = h
        self.device = dev
        self.tau = None

    def close(self):
        if getattr(self, "handle", None):
            call("abft_session_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def ws_handle(self):
        return lib.abft_session_ws(self.handle)

    def set_tau(self, tau):
        tau = np.broadcast_to(np.asarray(tau, np.float64), (self.F,)).copy()
        call("abft_session_set_tau", self.handle, _dptr(tau))
        self.tau = tau

    def set_golden(self, golden):
        self.golden = golden
        if golden is None:
            call("abft_session_set_golden", self.handle, None, 0)
        else:
            call("abft_session_set_golden", self.handle, golden.data_ptr(), golden.stride(0))

    def encode(self):
        ms = ctypes.c_double()
        with torch.cuda.device(self.device):
            call("abft_session_encode", self.handle, ctypes.byref(ms))
        return ms.value

    def baseline(self, repeats, graph=False):
        """repeats x F unprotected SGEMMs (the reference's pass_baseline); (device_ms, host_ms)."""
        dms, hms = ctypes.c_double(), ctypes.c_double()
        with torch.cuda.device(self.device):
            call("abft_session_baseline", self.handle, int(repeats), int(bool(graph)), ctypes.byref(dms),
                 ctypes.byref(hms))
        return dms.value, hms.value

    def baseline_monolithic(self, repeats, graph=False):
        """repeats x one unprotected SGEMM of the whole tile (no fragments); (device_ms, host_ms)."""
        dms, hms = ctypes.c_double(), ctypes.c_double()
        with torch.cuda.device(self.device):
            call("abft_session_baseline_monolithic", self.handle, int(repeats), int(bool(graph)), ctypes.byref(dms),
                 ctypes.byref(hms))
        return dms.value, hms.value

    def _args(self, mode, zone, add_delta, base_seed, rank, repeats, correct, log, profile=False, graph=False,
              seed_scheme="reference"):
        if correct not in ("inloop", "drain"):
            raise ValueError(f"correct must be 'inloop' or 'drain', not {correct!r}")
        if seed_scheme not in ("reference", "tile"):
            raise ValueError(f"seed_scheme must be 'reference' or 'tile', not {seed_scheme!r}")
        lo, hi = host.swifi_zone_range(zone)
        a = OnlineArgs()
        a.mode = host.MODES[mode] if isinstance(mode, str) else int(mode)
        a.zone_lo, a.zone_hi = lo, hi
        a.add_delta = float(add_delta)
        a.base_seed = int(base_seed)
        a.rank = int(rank)
        a.repeats = int(repeats)
        a.correct_mode = CORRECT_DRAIN if correct == "drain" else CORRECT_INLOOP
        a.log = int(bool(log))
        a.profile = int(bool(profile))
        a.graph = int(bool(graph))
        a.seed_scheme = 1 if seed_scheme == "tile" else 0
        return a

    @staticmethod
    def _result(r):
        return dict(device_ms=r.device_ms, host_ms=r.host_ms, cm=list(r.cm), n_restored=r.n_restored,
                    kernel_launches=r.kernel_launches, verify_launches=r.verify_launches,
                    verify_ms_sum=r.verify_ms_sum, verify_ms_max=r.verify_ms_max)

    def online(self, mode="none", zone="any", add_delta=ADD_FAULT_DELTA, base_seed=0, rank=0, repeats=1,
               correct="inloop", log=False, profile=False, graph=False, seed_scheme="reference"):
        """repeats protected iterations; returns timings, confusion matrix and restore count.

        profile=True brackets every verify launch with CUDA events on the verify
        stream (verify_ms_sum / verify_ms_max in the result). graph=True replays
        the loop as a CUDA graph (captured on first use for this shape).
        """
        if self.tau is None:
            raise RuntimeError("set_tau() first")
        a = self._args(mode, zone, add_delta, base_seed, rank, repeats, correct, log, profile, graph, seed_scheme)
        r = OnlineResult()
        with torch.cuda.device(self.device):
            call("abft_session_online", self.handle, ctypes.byref(a), ctypes.byref(r))
        return self._result(r)

    def run_host(self, hA, hB, hC, mode="none", zone="any", add_delta=ADD_FAULT_DELTA, base_seed=0, rank=0,
                 repeats=1, correct="inloop", profile=False):
        """End to end from host memory: hA and hB are copied into this session's
        A and B (overwriting them), then the checksums are encoded and the
        protected loop runs; the final C lands in hC. Pinned host tensors let
        the copies overlap the work."""
        for t in (hA, hB, hC):
            if t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError("host tensors must be contiguous float32 CPU tensors")
        a = self._args(mode, zone, add_delta, base_seed, rank, repeats, correct, False, profile)
        r = OnlineResult()
        e2e = ctypes.c_double()
        with torch.cuda.device(self.device):
            call("abft_session_run_host", self.handle, hA.data_ptr(), hB.data_ptr(), hC.data_ptr(), ctypes.byref(a),
                 ctypes.byref(r), ctypes.byref(e2e))
        out = self._result(r)
        out["e2e_ms"] = e2e.value
        return out

    def run_host_steps(self, hAs, hBs, hCs, base_seeds, mode="none", zone="any", add_delta=ADD_FAULT_DELTA, rank=0,
                       repeats=1, correct="inloop"):
        """Several end-to-end steps in one call, step k on (hAs[k], hBs[k]) with
        base_seeds[k], its final C into hCs[k] (entries may repeat a tensor).
        Results equal separate run_host calls on the same inputs; the copies of
        step k+1's inputs overlap step k's work (the session keeps a second
        device copy of A and B for that). Returns (per-step results, total
        e2e ms)."""
        n = len(base_seeds)
        if not (len(hAs) == len(hBs) == len(hCs) == n) or n < 1:
            raise ValueError("one hA, hB, hC per step and at least one step")
        for t in list(hAs) + list(hBs) + list(hCs):
            if t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError("host tensors must be contiguous float32 CPU tensors")
        a = self._args(mode, zone, add_delta, 0, rank, repeats, correct, False)
        P = ctypes.c_void_p * n
        pa = P(*[t.data_ptr() for t in hAs])
        pb = P(*[t.data_ptr() for t in hBs])
        pc = P(*[t.data_ptr() for t in hCs])
        seeds = (ctypes.c_uint64 * n)(*[int(x) for x in base_seeds])
        res = (OnlineResult * n)()
        e2e = ctypes.c_double()
        with torch.cuda.device(self.device):
            call("abft_session_run_host_steps", self.handle, n, pa, pb, pc, ctypes.byref(a), seeds, res,
                 ctypes.byref(e2e))
        return [self._result(r) for r in res], e2e.value

    def read_log(self, it_count):
        n = it_count * self.F
        ec = np.zeros(n, np.int32)
        er = np.zeros(n, np.int32)
        rd = np.zeros(n, np.float64)
        call("abft_ws_read_log", self.ws_handle, int(it_count), ec.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
             er.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), _dptr(rd))
        return ec.reshape(it_count, self.F), er.reshape(it_count, self.F), rd.reshape(it_count, self.F)

    def read_injections(self, it_count):
        inj = np.zeros(4 * it_count, np.int32)
        ba = np.zeros(2 * it_count, np.float32)
        call("abft_session_read_injections", self.handle, int(it_count),
             inj.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), ba.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return inj.reshape(it_count, 4), ba.reshape(it_count, 2)
