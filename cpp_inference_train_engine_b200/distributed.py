"""Data-parallel plumbing of the GRPO step: one process (rank) per GPU.

The rollout groups of a step are split evenly over the ranks, whole groups per rank
(``rollout_shard``), so group advantages stay local and a rank's rollout i is global rollout
``rank * R + i``. Every rank runs its own rollouts, teacher-forced passes and backward; the
engine divides each token's coefficient by the global rollout count, sums gradients and the
loss/KL scalars with an NCCL all-reduce over NVLink and ORs the "any non-zero advantage" flag
before the replicated AdamW (the reference's single-process update, trainer.cpp:784-891, with
its gradient sum split over ranks). The NCCL unique id reaches the ranks over a plain TCP
rendezvous served by rank 0 (``init_comm``), the host-side equivalent of what a C++ trainer
does with ``mm_cuda_nccl_unique_id``; no torch.distributed is involved.
"""
from __future__ import annotations

import os
import socket
import struct
import time


def rollout_shard(n_rollouts: int, group: int, rank: int, world: int) -> slice:
    """Rollouts [rank * R, (rank + 1) * R) with R = n_rollouts / world, whole groups only."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if group < 1 or n_rollouts % group:
        raise ValueError("rollouts must form whole groups")
    if n_rollouts % world or (n_rollouts // world) % group:
        raise ValueError("rollouts must split into whole groups per rank")
    R = n_rollouts // world
    return slice(rank * R, (rank + 1) * R)


def rendezvous_endpoint(addr: str | None = None, port: int | None = None) -> tuple[str, int]:
    """Where rank 0 serves the NCCL unique id: ``addr``/``port`` when given, else
    MM_RENDEZVOUS_ADDR / MM_RENDEZVOUS_PORT, else MASTER_ADDR and MASTER_PORT + 1 (the
    launcher's own rendezvous keeps MASTER_PORT)."""
    addr = addr or os.environ.get("MM_RENDEZVOUS_ADDR") or os.environ.get("MASTER_ADDR", "127.0.0.1")
    if port is None:
        if "MM_RENDEZVOUS_PORT" in os.environ:
            port = int(os.environ["MM_RENDEZVOUS_PORT"])
        elif "MASTER_PORT" in os.environ:
            port = int(os.environ["MASTER_PORT"]) + 1
        else:
            raise ValueError("no rendezvous port: set MM_RENDEZVOUS_PORT or MASTER_PORT")
    return addr, int(port)


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = b""
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("rendezvous peer closed the connection")
        buf += chunk
    return buf


def exchange_unique_id(rank: int, world: int, make_id, addr: str | None = None, port: int | None = None,
                       timeout: float = 300.0) -> bytes:
    """Every rank returns rank 0's ``make_id()`` (128 bytes), over plain TCP: rank 0 listens on
    the rendezvous endpoint and answers each other rank's connection with the id. A rank that
    does not arrive within ``timeout`` seconds turns into a RuntimeError on the ranks waiting
    for it, not a hang."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    host, prt = rendezvous_endpoint(addr, port)
    deadline = time.monotonic() + timeout
    if rank == 0:
        uid = bytes(make_id())
        if len(uid) != 128:
            raise RuntimeError("NCCL unique id must be 128 bytes")
        if world == 1:
            return uid
        with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as srv:
            srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            srv.bind((host, prt))
            srv.listen(world)
            served = set()
            while len(served) < world - 1:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise RuntimeError(f"rendezvous: {world - 1 - len(served)} rank(s) did not join "
                                       f"within {timeout:.0f} s")
                srv.settimeout(left)
                try:
                    conn, _ = srv.accept()
                except socket.timeout:
                    continue
                with conn:
                    conn.settimeout(max(deadline - time.monotonic(), 1.0))
                    peer = struct.unpack("<i", _recv_exact(conn, 4))[0]
                    if not 0 < peer < world or peer in served:
                        raise RuntimeError(f"rendezvous: unexpected rank {peer}")
                    conn.sendall(uid)
                    served.add(peer)
        return uid
    while True:
        left = deadline - time.monotonic()
        if left <= 0:
            raise RuntimeError(f"rendezvous: rank 0 did not answer at {host}:{prt} within {timeout:.0f} s")
        try:
            with socket.create_connection((host, prt), timeout=min(left, 5.0)) as c:
                c.settimeout(max(deadline - time.monotonic(), 1.0))
                c.sendall(struct.pack("<i", rank))
                return _recv_exact(c, 128)
        except (ConnectionRefusedError, socket.timeout, OSError):
            time.sleep(0.05)


def init_comm(execution, rank: int, world: int, addr: str | None = None, port: int | None = None,
              timeout: float = 300.0) -> None:
    """Bootstraps the execution's NCCL communicator (mm_cuda_init_comm): the unique id travels
    from rank 0 over the TCP rendezvous of ``exchange_unique_id`` (no torch.distributed)."""
    from .engine import CudaExecution
    uid = exchange_unique_id(rank, world, CudaExecution.nccl_unique_id, addr, port, timeout)
    execution.init_comm(rank, world, uid)
