"""Multi-GPU plumbing without torch: NCCL communicator rendezvous.

One process per GPU (launched e.g. by torchrun, which sets RANK, WORLD_SIZE,
LOCAL_RANK, MASTER_ADDR, MASTER_PORT). Rank 0 creates the 128-byte NCCL
unique id through the C ABI and serves it to the other ranks over a plain TCP
socket on MASTER_ADDR:(MASTER_PORT + 7); every rank then calls gpb_comm_init.
All data-path collectives (all-gather of packed column tiles, all-reduce of
dot products) run inside the CUDA library on the provider's stream.
"""
from __future__ import annotations

import ctypes as C
import os
import socket
import time

import numpy as np

from . import _lib

ID_BYTES = 128
PORT_OFFSET = 7


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) owned by `rank` (same rule as the C++ engine)."""
    return (n * rank) // world, (n * (rank + 1)) // world


def exchange_id(payload: bytes | None, rank: int, world: int, addr: str, port: int,
                timeout_s: float = 180.0) -> bytes:
    """Rank 0 serves `payload` to world-1 peers; other ranks fetch it."""
    deadline = time.monotonic() + timeout_s
    if rank == 0:
        assert payload is not None and len(payload) == ID_BYTES
        srv = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        srv.bind((addr, port))
        srv.listen(max(world - 1, 1))
        srv.settimeout(1.0)
        served = 0
        try:
            while served < world - 1:
                if time.monotonic() > deadline:
                    raise TimeoutError(f"rendezvous: only {served} of {world - 1} ranks connected")
                try:
                    conn, _ = srv.accept()
                except socket.timeout:
                    continue
                with conn:
                    conn.sendall(payload)
                served += 1
        finally:
            srv.close()
        return payload
    while True:
        try:
            with socket.create_connection((addr, port), timeout=5.0) as s:
                buf = b""
                while len(buf) < ID_BYTES:
                    chunk = s.recv(ID_BYTES - len(buf))
                    if not chunk:
                        break
                    buf += chunk
                if len(buf) == ID_BYTES:
                    return buf
        except OSError:
            pass
        if time.monotonic() > deadline:
            raise TimeoutError("rendezvous: could not fetch the communicator id from rank 0")
        time.sleep(0.2)


class Communicator:
    """A gpb_comm handle (NCCL communicator for this rank's GPU)."""

    def __init__(self, rank: int, world: int, device: int, uid: bytes):
        self.rank, self.world, self.device = rank, world, device
        buf = (C.c_uint8 * ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        _lib.call("gpb_comm_init", C.cast(buf, C.c_void_p), world, rank, device, C.byref(h))
        self.handle = h.value

    @classmethod
    def from_env(cls, device: int | None = None) -> "Communicator":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        device = int(os.environ.get("LOCAL_RANK", "0")) if device is None else device
        addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
        port = int(os.environ.get("MASTER_PORT", "29500")) + PORT_OFFSET
        uid = None
        if rank == 0:
            raw = (C.c_uint8 * ID_BYTES)()
            _lib.call("gpb_comm_unique_id", C.cast(raw, C.c_void_p))
            uid = bytes(raw)
        uid = exchange_id(uid, rank, world, addr, port)
        return cls(rank, world, device, uid)

    @property
    def h(self) -> C.c_void_p:
        return C.c_void_p(self.handle)

    def barrier(self) -> None:
        _lib.call("gpb_comm_barrier", self.h)

    def allreduce_max(self, value: float) -> float:
        v = C.c_double(value)
        _lib.call("gpb_comm_allreduce_max_f64", self.h, C.byref(v))
        return v.value

    def allreduce_sum(self, values) -> np.ndarray:
        a = np.ascontiguousarray(values, dtype=np.float64).copy()
        _lib.call("gpb_comm_allreduce_sum_f64", self.h, C.c_void_p(a.ctypes.data), a.size)
        return a

    def benchmark_sharded_forward(self, prov, vd, od, t, warmup, steps, r0, r1):
        step_ms = np.zeros(steps)
        kern_ms = np.zeros(steps)
        launches = np.zeros(steps, dtype=np.int64)
        _lib.call("gpb_benchmark_forward_sharded", prov.h, self.h, vd.cptr, t, warmup, steps, 1,
                  C.c_void_p(step_ms.ctypes.data), C.c_void_p(kern_ms.ctypes.data),
                  C.c_void_p(launches.ctypes.data))
        return step_ms, kern_ms, launches

    def matvec_sharded(self, prov, V_local: np.ndarray) -> np.ndarray:
        """(K + noise I) V for this rank's rows: V_local [t][n_local] host
        array of this rank's rows, returns the same rows of the product (the
        mBCG iteration's product, column side all-gathered over NCCL)."""
        from .provider import DeviceBuffer
        V_local = np.ascontiguousarray(V_local, np.float32)
        vd = DeviceBuffer.from_host(V_local, prov.device)
        od = DeviceBuffer(V_local.shape, prov.device)
        _lib.call("gpb_matvec_sharded", prov.h, self.h, od.cptr, vd.cptr, V_local.shape[0])
        return od.download()

    def e2e_sharded(self, prov, Vc: np.ndarray, t: int, r0: int, r1: int, flops_total: float,
                    reps: int = 2) -> float:
        """Host V in, this rank's output rows back to the host; max over ranks."""
        from .provider import DeviceBuffer, pinned
        vd = DeviceBuffer(Vc.shape, prov.device)
        od = DeviceBuffer((t, r1 - r0), prov.device)
        Vc = np.ascontiguousarray(Vc)
        out_h = np.empty((t, r1 - r0), np.float32)
        with pinned(Vc, out_h):
            self.barrier()
            t0 = time.perf_counter()
            for _ in range(reps):
                vd.upload(Vc)
                prov.forward_matvec_rows(od, vd, t, r0, r1)
                prov.synchronize()
                od.download(out_h)
            dt = (time.perf_counter() - t0) / reps
        dt = self.allreduce_max(dt)
        return flops_total / dt / 1e12

    def close(self) -> None:
        if getattr(self, "handle", None):
            _lib.lib().gpb_comm_destroy(self.h)
            self.handle = None
