"""Multi-GPU sgemm / dgemm: C sharded by row blocks, B broadcast over NVLink.

The reference drives several GPUs only as independent devices
(examples/init-two-gpus/init-two-gpus.js); this module adds the sharded GEMM
of its multi-GPU target on top of the C ABI's communicator (wg_comm_*,
wgblas_b200/csrc/shard.cu). One process per GPU: every rank holds its row
block of op(A) and of C resident on its GPU (scattered once), and B lives on
the root; each call sends B in column panels to the other ranks (a copy-engine
chain over NVLink, or ncclBroadcast), the GEMM of each panel starting as soon
as the panel has arrived.

The host-side planning here (``plan_rows``, ``row_block``, ``place_rows``) is
pure Python/numpy and is what the CPU multi-process tests check.
"""
from __future__ import annotations

import ctypes as ct
import os

import numpy as np

from . import _native as nat
from ._runtime import Device
from .classes import GpuMatrix


def plan_rows(m: int, nranks: int, align: int = 128) -> list[int]:
    """Row offsets (nranks + 1 entries) splitting m rows into contiguous blocks.

    Blocks are multiples of `align` rows (the tensor-core kernels' tile height)
    except the last non-empty one, and differ by at most `align` rows."""
    if nranks < 1:
        raise ValueError("nranks must be >= 1")
    units = -(-m // align) if m > 0 else 0
    base, extra = divmod(units, nranks)
    offs = [0]
    for r in range(nranks):
        u = base + (1 if r < extra else 0)
        offs.append(min(m, offs[-1] + u * align))
    offs[-1] = m
    return offs


def row_block(X: np.ndarray, rows: int, cols: int, ld: int, r0: int, r1: int, trans: bool) -> tuple[np.ndarray, int]:
    """Rows [r0, r1) of op(X) for a column-major X (rows x cols of op(X)), as a
    dense column-major block of op(X)'s orientation: returns (block, ld_block).

    Without trans, op(X) = X and the block is X[r0:r1, :] (ld = r1 - r0); with
    trans, op(X) = X^T and the block is X[:, r0:r1] stored as its own column-major
    (cols x (r1-r0)) matrix, so the caller keeps trans set (ld = cols)."""
    mr = r1 - r0
    if not trans:
        out = np.empty(max(mr * cols, 1), X.dtype)[: mr * cols]
        for j in range(cols):
            out[j * mr:(j + 1) * mr] = X[r0 + j * ld: r1 + j * ld]
        return out, max(mr, 1)
    out = np.empty(max(cols * mr, 1), X.dtype)[: cols * mr]
    for i in range(mr):
        out[i * cols:(i + 1) * cols] = X[(r0 + i) * ld: (r0 + i) * ld + cols]
    return out, max(cols, 1)


def place_rows(C_full: np.ndarray, ldc: int, block: np.ndarray, ld_block: int, r0: int, r1: int, n: int) -> None:
    """Writes a dense column-major row block back into rows [r0, r1) of C_full."""
    mr = r1 - r0
    for j in range(n):
        C_full[r0 + j * ldc: r1 + j * ldc] = block[j * ld_block: j * ld_block + mr]


def _prefer_bundled_nccl() -> None:
    """Points the library's NCCL loader at the NCCL that ships with torch's CUDA
    wheels when present (WGBLAS_NCCL_LIBRARY, unless already set). Two NCCLs in
    one process share the soname libnccl.so.2: whichever loads first serves both
    this library and torch, and torch's CUDA library needs its own (newer) one."""
    if os.environ.get("WGBLAS_NCCL_LIBRARY"):
        return
    try:
        import importlib.util

        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return
    for base in (spec.submodule_search_locations or []) if spec else []:
        cand = os.path.join(base, "lib", "libnccl.so.2")
        if os.path.exists(cand):
            os.environ["WGBLAS_NCCL_LIBRARY"] = cand
            return


class Comm:
    """A communicator joining one device handle to the other ranks' (wg_comm)."""

    def __init__(self, device: Device, nranks: int, rank: int, unique_id: bytes, timeout_ms: int = 60000):
        _prefer_bundled_nccl()
        self.device = device
        self.nranks = nranks
        self.rank = rank
        h = nat.c_comm_p()
        nat.check(nat.lib.wg_comm_init_rank(device.handle, nranks, rank, unique_id, len(unique_id), timeout_ms,
                                            ct.byref(h)))
        self._h = h
        self._host_buffers = None  # gemm_sharded_host's device buffers

    def _free_host_buffers(self) -> None:
        if self._host_buffers is not None:
            for g in self._host_buffers[1:]:
                if g is not None:
                    g.destroy()
            self._host_buffers = None

    @staticmethod
    def unique_id() -> bytes:
        _prefer_bundled_nccl()
        buf = ct.create_string_buffer(128)
        nat.check(nat.lib.wg_comm_unique_id(buf, 128))
        return buf.raw

    @property
    def handle(self):
        if self._h is None:
            raise RuntimeError("communicator destroyed")
        return self._h

    def wait(self) -> None:
        nat.check(nat.lib.wg_comm_wait(self.handle))

    def abort(self) -> None:
        if self._h is not None:
            nat.lib.wg_comm_abort(self._h)

    def destroy(self) -> None:
        if self._h is not None:
            self._free_host_buffers()
            nat.lib.wg_comm_destroy(self._h)
            self._h = None


def comm_from_torch(device: Device, timeout_ms: int = 60000) -> Comm:
    """Creates the communicator of a torch.distributed job (any backend; the
    128-byte id travels through it)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(), dist.get_world_size()
    box = [Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return Comm(device, world, rank, box[0], timeout_ms)


def _ptr(g: GpuMatrix) -> ct.c_void_p:
    return ct.c_void_p(g.device_ptr())


def gemm_sharded(comm: Comm, transA: bool, transB: bool, m_local: int, n: int, k: int, alpha, A_local: GpuMatrix,
                 B: GpuMatrix | None, beta, C_local: GpuMatrix, root: int = 0, panel_cols: int = 0,
                 ldb: int | None = None) -> None:
    """Queues this rank's C_local := alpha*op(A_local)*op(B) + beta*C_local with B
    sent from `root` (column-major GpuMatrix operands). B is read on the root
    only: other ranks may pass None (then give ``ldb``, the root's leading
    dimension) and receive root's B into the communicator's buffer. dtype follows
    the operands (float32 -> sgemm)."""
    f64 = np.dtype(C_local.dtype) == np.float64
    fn = nat.lib.wg_dgemm_sharded if f64 else nat.lib.wg_sgemm_sharded
    al, be = (float(alpha), float(beta)) if f64 else (np.float32(alpha), np.float32(beta))
    if ldb is None:
        if B is None:
            raise ValueError("ldb is required when B is None")
        ldb = B.lda
    nat.check(fn(comm.handle, int(bool(transA)), int(bool(transB)), m_local, n, k, al,
                 _ptr(A_local) if m_local else None, A_local.lda, _ptr(B) if B is not None else None, ldb, root, be,
                 _ptr(C_local) if m_local else None, C_local.lda, panel_cols))


def gemm_sharded_host(comm: Comm, transA: bool, transB: bool, m_local: int, n: int, k: int, alpha,
                      A_local: np.ndarray, B: np.ndarray | None, ldb: int, beta, C_local: np.ndarray,
                      row_offsets: list[int], root: int = 0, panel_cols: int = 0,
                      out: np.ndarray | None = None) -> np.ndarray | None:
    """The sharded GEMM on host arrays, the typed-array counterpart of
    ``gemm_sharded`` (as the reference's sgemm takes typed arrays and returns a
    new C, src/sgemm/sgemm.mjs:151-262): every rank uploads its row block of
    op(A) (dense column-major, ``row_block``'s layout: m_local x k, or k x m_local
    with transA) and of C (m_local x n, ld m_local); the root uploads B (its
    stored matrix, leading dimension ldb; other ranks pass None). The product
    runs sharded, the row blocks are gathered on the root, and the root returns
    the full column-major C (m x n, ld m; into ``out`` when given, e.g. a
    page-locked array); other ranks return None. The device buffers of the last
    shape stay on the communicator for the next call (Comm.destroy frees them).
    Collective: every rank must call it."""
    dev = comm.device
    dt = np.dtype(C_local.dtype)
    m = row_offsets[-1]
    a_rows, a_cols = (k, m_local) if transA else (m_local, k)
    b_rows, b_cols = (n, k) if transB else (k, n)
    # Device buffers of the last shape are kept on the communicator (freed by
    # destroy()): allocating and freeing a few GiB per call would dominate it.
    key = (dt.str, a_rows, a_cols, m_local, n, b_rows, b_cols, ldb, m, comm.rank == root)
    cached = comm._host_buffers
    if cached is None or cached[0] != key:
        comm._free_host_buffers()
        GA = GpuMatrix.empty(dev, a_rows, a_cols, a_rows, "column-major", dt) if m_local else None
        GC = GpuMatrix.empty(dev, m_local, n, m_local, "column-major", dt) if m_local else None
        GB = GpuMatrix.empty(dev, b_rows, b_cols, ldb, "column-major", dt) if comm.rank == root else None
        GF = GpuMatrix.empty(dev, m, n, m, "column-major", dt) if comm.rank == root else None
        comm._host_buffers = cached = (key, GA, GC, GB, GF)
    _, GA, GC, GB, GF = cached
    if GA is not None:
        GA.write(A_local)
        GC.write(C_local)
    if GB is not None:
        GB.write(B)
    gemm_sharded(comm, transA, transB, m_local, n, k, alpha, GA, GB, beta, GC, root=root,
                 panel_cols=panel_cols, ldb=ldb)
    gather_rows(comm, GC, m_local, n, row_offsets, root=root, C_full=GF)
    dev.synchronize()
    comm.wait()
    dev.check()
    return GF.read(out) if GF is not None else None


def gather_rows(comm: Comm, C_local: GpuMatrix, m_local: int, n: int, row_offsets: list[int], root: int = 0,
                C_full: GpuMatrix | None = None) -> None:
    """Queues the gather of every rank's C rows into C_full on `root`."""
    f64 = np.dtype(C_local.dtype) == np.float64
    fn = nat.lib.wg_dgemm_gather_rows if f64 else nat.lib.wg_sgemm_gather_rows
    offs = (ct.c_int64 * len(row_offsets))(*row_offsets)
    nat.check(fn(comm.handle, _ptr(C_local) if m_local else None, m_local, n, C_local.lda, root,
                 _ptr(C_full) if C_full is not None else None, C_full.lda if C_full is not None else 0, offs))
