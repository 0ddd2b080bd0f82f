"""KV transfer on B200: PaceServe's ``KVhelper`` interface backed by one CUDA
kernel per move, plus LP -> HP block promotion over NVLink.

Reference interface (paceserve/kv_transfer/kv_utils.py:8-56):
``KVhelper(rank, model_config, cache_config, parallel_config)`` with
``add_model_runner``, ``reset_kv_cache``, ``get_kv_cache(seq, seq_manager)``
and ``insert_kv_cache(cached_content, kv_indices, device)``.  The reference
gathers a sequence's blocks with one fancy-index copy per layer into a CPU
tensor and scatters them back with one index-put per layer; here each
direction is a single gather/scatter kernel over all layers, reading or
writing page-locked host memory directly.

New capability (no reference counterpart): ``promote`` copies a request's
blocks from another GPU's cache -- the low-priority (LP) worker's -- into
free blocks of this worker's cache over NVLink P2P, either within one
process (peer access) or across processes (CUDA IPC handles exchanged as
``CacheExport`` records).
"""
from __future__ import annotations

import dataclasses
from typing import List, Optional, Sequence

import torch

from . import _C

kv_ops = _C.kv_transfer_ops


# ------------------------------------------------------------- helpers ----
def _ids_tensor(ids: Sequence[int] | torch.Tensor, device: torch.device) -> torch.Tensor:
    if isinstance(ids, torch.Tensor):
        return ids.to(device=device, dtype=torch.int32)
    return torch.tensor(list(ids), dtype=torch.int32, device=device)


def align_block_tables(num_src_blocks: int, dst_table: Sequence[int]) -> List[int]:
    """Destination blocks that receive `num_src_blocks` transferred blocks.

    Restates the rule of BaseWorker._insert_kv_cache
    (paceserve/worker/base_worker.py:262-277): the receiving worker allocates
    the sequence's blocks from its logical token count, which can be one block
    longer than what the sender holds (the extra logical token of a prefilled
    sequence, or a decode step whose block was allocated on one side only).
    In that case the last destination block is left out.
    """
    dst = list(dst_table)
    if len(dst) == num_src_blocks:
        return dst
    if len(dst) == num_src_blocks + 1:
        return dst[:-1]
    raise ValueError(
        f"block tables do not line up: {num_src_blocks} source blocks, {len(dst)} destination blocks")


def plan_promotion(src_tables: Sequence[Sequence[int]], free_blocks: Sequence[int]):
    """Concatenate the source block tables of the promoted requests and assign
    each block a free destination block, in order (as the destination's
    allocator hands out free blocks, base_block_space_manager.py:11-64).
    Returns (src_ids, dst_ids, per-request destination tables)."""
    need = sum(len(t) for t in src_tables)
    if need > len(free_blocks):
        raise ValueError(f"not enough free destination blocks: need {need}, have {len(free_blocks)}")
    src_ids, dst_ids, tables = [], [], []
    it = iter(free_blocks)
    for t in src_tables:
        d = [next(it) for _ in t]
        src_ids.extend(t)
        dst_ids.extend(d)
        tables.append(d)
    if len(set(src_ids)) != len(src_ids):
        raise ValueError("a source block appears twice")
    return src_ids, dst_ids, tables


# ------------------------------------------------------------ IPC export --
@dataclasses.dataclass
class CacheExport:
    """What another process needs to address a worker's per-layer KV caches."""

    handles: List[bytes]
    offsets: List[int]
    num_blocks: int
    block_bytes: int
    device: int
    shape: tuple
    dtype: str

    @property
    def num_layers(self) -> int:
        return len(self.handles)


def export_caches(caches: Sequence[torch.Tensor]) -> CacheExport:
    """CUDA IPC handles of a list of per-layer caches [num_blocks, ...]."""
    if not caches:
        raise ValueError("no caches to export")
    handles, offsets = [], []
    c0 = caches[0]
    for c in caches:
        if not (c.is_cuda and c.is_contiguous()):
            raise ValueError("caches must be contiguous CUDA tensors")
        if c.shape != c0.shape or c.dtype != c0.dtype or c.device != c0.device:
            raise ValueError("every layer's cache must share the first layer's shape, dtype "
                             "and device")
        h, off = kv_ops.ipc_get_handle(c)
        handles.append(bytes(h))
        offsets.append(int(off))
    return CacheExport(handles, offsets, int(c0.shape[0]),
                       int(c0[0].numel() * c0.element_size()) if c0.shape[0] else 0,
                       int(c0.device.index), tuple(c0.shape), str(c0.dtype))


class ImportedCaches:
    """Another process's caches mapped into this process on `device`."""

    def __init__(self, export: CacheExport, device: int):
        self.export = export
        self.device = int(device)
        self._bases: List[int] = []
        self.ptrs: List[int] = []
        try:
            opened = {}
            for h in export.handles:
                if h not in opened:  # layers may share one allocation
                    opened[h] = kv_ops.ipc_open_handle(h, self.device)
                    self._bases.append(opened[h])
            self.ptrs = [opened[h] + off for h, off in zip(export.handles, export.offsets)]
        except Exception:
            self.close()
            raise

    @property
    def num_blocks(self) -> int:
        return self.export.num_blocks

    def close(self) -> None:
        """Unmap the peer's caches (idempotent).  Synchronises this device first,
        so no copy still reading the mapping is in flight when it goes away.
        Not done implicitly on garbage collection, for the same reason."""
        bases, self._bases, self.ptrs = self._bases, [], []
        if bases:
            torch.cuda.synchronize(self.device)
        for b in bases:
            kv_ops.ipc_close_handle(b)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# Copy methods of promote()/push(): the SM kernels of pace_kv_copy_blocks, and
# the copy engines (pace_kv_copy_blocks_ce), which use no SM of either GPU.
METHOD_AUTO, METHOD_SIMT, METHOD_BULK, METHOD_COPY_ENGINE = 0, 1, 2, 3


class KVCopyError(RuntimeError):
    """A promotion copy skipped pairs or one of its waits expired."""


def check_copy_status(counter: torch.Tensor) -> None:
    """Synchronise with the copy that `counter` belongs to and raise KVCopyError
    if it counted out-of-range pairs or flagged an expired wait (bit 30) or a
    load still in flight after the drain (bit 29)."""
    v = int(counter.item())
    if v == 0:
        return
    timeout = bool(v & (1 << 30))
    drain = bool(v & (1 << 29))
    bad = v & ((1 << 29) - 1)
    parts = []
    if bad:
        parts.append(f"{bad} block pair(s) out of range were skipped")
    if timeout:
        parts.append("a bounded wait expired, the copy is incomplete")
    if drain:
        parts.append("a load was still in flight after the drain; do not trust this device")
    raise KVCopyError("KV block copy: " + "; ".join(parts))


def _counter(dev: torch.device, bad_pairs: Optional[torch.Tensor]) -> torch.Tensor:
    if bad_pairs is not None:
        return bad_pairs
    return torch.zeros(1, dtype=torch.int32, device=dev)


def _ids_for(method: int, ids, dev: torch.device):
    # the copy-engine path reads host ids; the kernels read device ids
    if method == METHOD_COPY_ENGINE:
        if isinstance(ids, torch.Tensor):
            return ids.to(device="cpu", dtype=torch.int32)
        return torch.tensor(list(ids), dtype=torch.int32)
    return _ids_tensor(ids, dev)


def promote(src, dst_caches: Sequence[torch.Tensor], src_block_ids, dst_block_ids,
            method: int = METHOD_AUTO, bad_pairs: Optional[torch.Tensor] = None,
            max_ctas: int = 0, wait_limit_ns: int = 0) -> torch.Tensor:
    """Pull blocks src_block_ids of `src` into dst_block_ids of `dst_caches`,
    on the destination GPU's current stream.  `src` is either a list of
    per-layer tensors (any GPU of this process) or an ImportedCaches.

    method: METHOD_SIMT / METHOD_BULK run a kernel on the destination GPU
    (max_ctas > 0 caps its CTAs, leaving SMs to the serving instance);
    METHOD_COPY_ENGINE queues copies on the copy engines and uses no SM.
    Returns the int32 counter of skipped pairs and wait flags (`bad_pairs`, or
    a new one), which check_copy_status() reads after the copy."""
    dev = dst_caches[0].device
    s = _ids_for(method, src_block_ids, dev)
    d = _ids_for(method, dst_block_ids, dev)
    bad = _counter(dev, bad_pairs)
    if isinstance(src, ImportedCaches):
        with torch.cuda.device(dev):
            kv_ops.copy_blocks_from_ptrs(src.ptrs, src.num_blocks, list(dst_caches), s, d, method,
                                         bad, max_ctas, wait_limit_ns)
    else:
        kv_ops.copy_blocks_p2p(list(src), list(dst_caches), s, d, method, False, bad, max_ctas,
                               wait_limit_ns)
    return bad


def push(src_caches: Sequence[torch.Tensor], dst, src_block_ids, dst_block_ids,
         method: int = METHOD_AUTO, bad_pairs: Optional[torch.Tensor] = None, max_ctas: int = 0,
         wait_limit_ns: int = 0) -> torch.Tensor:
    """Push blocks from this process's caches into `dst` (ImportedCaches of the
    receiving worker, or tensors), on the source GPU's current stream.  The
    kernel (or the copy engines) of the source GPU does the work, so the
    receiving GPU's SMs stay free for serving.  Returns the counter, as
    promote() does."""
    dev = src_caches[0].device
    s = _ids_for(method, src_block_ids, dev)
    d = _ids_for(method, dst_block_ids, dev)
    bad = _counter(dev, bad_pairs)
    if isinstance(dst, ImportedCaches):
        with torch.cuda.device(dev):
            kv_ops.copy_blocks_to_ptrs(list(src_caches), dst.ptrs, dst.num_blocks, s, d, method,
                                       bad, max_ctas, wait_limit_ns)
    else:
        kv_ops.copy_blocks_p2p(list(src_caches), list(dst), s, d, method, True, bad, max_ctas,
                               wait_limit_ns)
    return bad


def pair_ranks(world_size: int) -> List[tuple]:
    """LP -> HP pairs (0->1), (2->3), ...; an odd last rank has no partner."""
    return [(r, r + 1) for r in range(0, world_size - 1, 2)]


def exchange_exports(export: Optional[CacheExport], group=None) -> List[Optional[CacheExport]]:
    """All ranks' CacheExport (or None) through torch.distributed."""
    import torch.distributed as dist

    out: List[Optional[CacheExport]] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, export, group=group)
    return out


# --------------------------------------------------------------- KVhelper --
class KVhelper:
    """Drop-in for paceserve.kv_transfer.kv_utils.KVhelper (kv_utils.py:8-56)."""

    def __init__(self, rank, model_config, cache_config, parallel_config):
        self.rank = rank
        self.num_q_heads = model_config.get_num_q_heads(parallel_config)
        self.num_kv_heads = model_config.get_num_kv_heads(parallel_config)
        self.head_dim = model_config.get_head_size()
        self.dtype = model_config.dtype
        self.block_size = cache_config.block_size
        self.num_layers = model_config.get_num_layers(parallel_config)
        self.model_runner = None

    def add_model_runner(self, model_runner):
        self.model_runner = model_runner

    @property
    def gpu_cache(self) -> List[torch.Tensor]:
        return self.model_runner.attention_backend_wrapper.gpu_cache

    def _block_shape(self):
        return (2, self.block_size, self.num_kv_heads, self.head_dim)

    def reset_kv_cache(self, num_gpu_blocks):
        """kv_utils.py:29-31: zero-filled per-layer caches."""
        for i in range(self.num_layers):
            self.gpu_cache[i] = torch.zeros(num_gpu_blocks, *self._block_shape(), dtype=self.dtype,
                                            device="cuda")

    def get_kv_cache(self, seq, seq_manager):
        """kv_utils.py:33-47: (CPU tensor [L, n, 2, bs, kv_heads, hd], block table).
        One gather kernel writes all layers straight into page-locked memory."""
        try:
            kv_page_indices = seq_manager._get_block_table(seq)
        except Exception:
            kv_page_indices = None
        if not kv_page_indices:
            return torch.zeros(self.num_layers, 1, *self._block_shape(), dtype=self.dtype), [0]
        cache = self.gpu_cache
        out = torch.empty(self.num_layers, len(kv_page_indices), *self._block_shape(),
                          dtype=self.dtype, pin_memory=True)
        ids = _ids_tensor(kv_page_indices, cache[0].device)
        kv_ops.gather_blocks(list(cache[: self.num_layers]), ids, out)
        torch.cuda.current_stream(cache[0].device).synchronize()
        return out, kv_page_indices

    def insert_kv_cache(self, cached_content, kv_indices, device):
        """kv_utils.py:49-56: scatter [L, n, ...] onto blocks kv_indices of every
        layer; True on success, False (with the error printed) otherwise."""
        try:
            cache = self.gpu_cache
            src = cached_content
            if isinstance(src, (list, tuple)):
                src = torch.stack([torch.as_tensor(x) for x in src])
            if not src.is_cuda and not src.is_pinned():
                src = src.pin_memory()
            src = src.contiguous()
            ids = _ids_tensor(kv_indices, cache[0].device)
            kv_ops.scatter_blocks(src, list(cache[: self.num_layers]), ids)
            torch.cuda.current_stream(cache[0].device).synchronize()
            return True
        except Exception as e:  # same contract as the reference
            print(f"error during insert kv cache: {e}")
            return False

    # -- new: NVLink promotion -------------------------------------------
    def export_cache(self) -> CacheExport:
        return export_caches(self.gpu_cache[: self.num_layers])

    def promote_from(self, source, src_block_ids, dst_block_ids, method: int = METHOD_AUTO,
                     max_ctas: int = 0) -> None:
        """Copy a promoted request's blocks from `source` (an ImportedCaches of the
        LP worker or its tensors) into this worker's blocks dst_block_ids, and
        wait for it (like get_kv_cache/insert_kv_cache).  Raises KVCopyError if
        pairs were out of range or a wait expired."""
        bad = promote(source, self.gpu_cache[: self.num_layers], src_block_ids, dst_block_ids,
                      method, max_ctas=max_ctas)
        check_copy_status(bad)

    def push_to(self, dest, src_block_ids, dst_block_ids, method: int = METHOD_SIMT) -> None:
        """Run on the LP worker: copy a promoted request's blocks src_block_ids of
        this worker's cache into blocks dst_block_ids of `dest` (an ImportedCaches
        of the HP worker's export) over NVLink, with this GPU's SMs (or, with
        METHOD_COPY_ENGINE, its copy engines), and wait for it.  The HP GPU keeps
        all its SMs for serving: on B200 a 1.1 GB promotion pushed this way slowed
        the HP instance's 32-layer chain by 10 % (pulling on the HP GPU: 98 %).
        Raises KVCopyError if pairs were out of range or a wait expired."""
        bad = push(self.gpu_cache[: self.num_layers], dest, src_block_ids, dst_block_ids, method)
        check_copy_status(bad)
