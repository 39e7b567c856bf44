"""KV caches: paged pool with prefix sharing, and per-slot contiguous cache.

API parity with astrai/inference/core/cache.py:10-525 (``page_hash``,
``Allocator``, ``PrefixCache``, ``PagePool``, ``TaskTable``, ``Storage``,
``CacheView``, ``KVCache``, ``PageCacheView``, ``PageCache``,
``ContiguousCacheView``, ``ContiguousCache``).

Layout and execution differ:

* One storage layout for both caches: per layer ``[n_pages, Hkv, page_size,
  128]`` so the keys of one head inside a page are contiguous. The contiguous
  cache is the same storage with one page per batch slot
  (``page_size = max_seq_len``), so both run the same kernels.
* Views carry per-row lengths on the device (``lens`` int32, the number of
  cached keys after this step) and an int32 page table; attention layers call
  :meth:`CacheView.attend` / :meth:`CacheView.attend_qkv`, which write the new
  K/V (one kernel) and run attention reading the pages in-kernel: the paged
  split-KV decode kernel for one new token, the flash kernel for prefill
  (over the gathered prefix when pages were shared). Nothing is gathered per
  decode step.
* ``page_hash`` chains page hashes (the hash of page i covers pages 0..i), so
  a hit on page i implies the whole prefix matched; a per-page hash would let
  equal page contents after different prefixes share KV that differs.
* A prompt never hits all of its pages: at least its last token is
  recomputed, so prefill always produces the logits of the last prompt token.
"""

from __future__ import annotations

import heapq
import math
import threading
from abc import ABC, abstractmethod
from collections import OrderedDict
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
from torch import Tensor

_MASK64 = 0xFFFFFFFFFFFFFFFF
HEAD_DIM = 128
KERNEL_HEAD_DIMS = (64, 128)  # head sizes the cache kernels (write, gather, decode) support


def _page_hash_step(prev: int, token_ids: Sequence[int], start: int, end: int) -> int:
    h = (prev * 1000003 + 0x9E3779B97F4A7C15) & _MASK64
    for i in range(start, end):
        h = (h * 31 + int(token_ids[i]) + 1) & _MASK64
    return h


def page_hash(token_ids: Sequence[int], page_idx: int, page_size: int) -> int:
    """Chained hash of pages ``0..page_idx`` of ``token_ids``."""
    h = 0
    for i in range(page_idx + 1):
        s = i * page_size
        h = _page_hash_step(h, token_ids, s, min(s + page_size, len(token_ids)))
    return h


def _page_hashes(token_ids: Sequence[int], n_pages: int, page_size: int) -> List[int]:
    out, h = [], 0
    for i in range(n_pages):
        s = i * page_size
        h = _page_hash_step(h, token_ids, s, min(s + page_size, len(token_ids)))
        out.append(h)
    return out


class Allocator:
    """Page allocator: lowest free index first, refcounts, LRU of cached pages.

    A page whose refcount drops to 0 either returns to the free set or (when
    its content is still addressable by hash) waits in the LRU, from which it
    is evicted (``on_evict(idx)``) only when no free page is left.
    """

    def __init__(self, n_pages: int):
        self.n_pages = n_pages
        self._free: List[int] = list(range(n_pages))
        heapq.heapify(self._free)
        self._refs: List[int] = [0] * n_pages
        self._lru: "OrderedDict[int, None]" = OrderedDict()
        self.on_evict: Optional[Callable[[int], None]] = None
        self._lock = threading.Lock()

    def alloc(self) -> int:
        with self._lock:
            if self._free:
                idx = heapq.heappop(self._free)
            elif self._lru:
                idx, _ = self._lru.popitem(last=False)
                if self.on_evict:
                    self.on_evict(idx)
            else:
                return -1
            self._refs[idx] = 1
            return idx

    def free(self, idx: int, keep_cached: bool = False) -> None:
        with self._lock:
            self._refs[idx] -= 1
            if self._refs[idx] == 0:
                if keep_cached:
                    self._lru[idx] = None
                else:
                    heapq.heappush(self._free, idx)

    def inc_ref(self, idx: int) -> None:
        with self._lock:
            self._refs[idx] += 1
            self._lru.pop(idx, None)

    def ref_count(self, idx: int) -> int:
        with self._lock:
            return self._refs[idx]

    def touch(self, idx: int) -> None:
        with self._lock:
            if idx in self._lru:
                self._lru.move_to_end(idx)

    @property
    def num_free(self) -> int:
        with self._lock:
            return len(self._free) + len(self._lru)


class PrefixCache:
    """Chained page hash -> physical page."""

    def __init__(self, page_size: int):
        self._page_size = page_size
        self._page_to_hash: Dict[int, int] = {}
        self._hash_to_page: Dict[int, int] = {}
        self._lock = threading.Lock()

    def evict(self, idx: int) -> None:
        with self._lock:
            h = self._page_to_hash.pop(idx, None)
            if h is not None and self._hash_to_page.get(h) == idx:
                del self._hash_to_page[h]

    def has_page(self, idx: int) -> bool:
        with self._lock:
            return idx in self._page_to_hash

    def lookup(self, token_ids: Sequence[int], max_pages: Optional[int] = None) -> List[int]:
        full = len(token_ids) // self._page_size
        if max_pages is not None:
            full = min(full, max_pages)
        hits: List[int] = []
        with self._lock:
            for h in _page_hashes(token_ids, full, self._page_size):
                p = self._hash_to_page.get(h)
                if p is None:
                    break
                hits.append(p)
        return hits

    def record(self, page_idx: int, token_ids: Sequence[int], logical_page_idx: int) -> None:
        self.record_hash(page_idx, page_hash(token_ids, logical_page_idx, self._page_size))

    def record_hash(self, page_idx: int, h: int) -> None:
        with self._lock:
            old = self._page_to_hash.pop(page_idx, None)
            if old is not None and self._hash_to_page.get(old) == page_idx:
                del self._hash_to_page[old]
            self._page_to_hash[page_idx] = h
            self._hash_to_page[h] = page_idx


class PagePool:
    """Allocator + PrefixCache: cached pages survive their last owner."""

    def __init__(self, allocator: Allocator, prefix: PrefixCache):
        self._alloc = allocator
        self._prefix = prefix
        self._alloc.on_evict = prefix.evict

    @property
    def allocator(self) -> Allocator:
        return self._alloc

    @property
    def prefix(self) -> PrefixCache:
        return self._prefix

    def alloc(self) -> int:
        return self._alloc.alloc()

    def free(self, idx: int) -> None:
        keep = self._prefix.has_page(idx)
        self._alloc.free(idx, keep_cached=keep)

    def inc_ref(self, idx: int) -> None:
        self._alloc.inc_ref(idx)

    def lookup(self, token_ids: Sequence[int], max_pages: Optional[int] = None) -> List[int]:
        hits = self._prefix.lookup(token_ids, max_pages)
        for p in hits:
            self._alloc.touch(p)
        return hits

    def record(self, page_idx: int, token_ids: Sequence[int], logical_page_idx: int) -> None:
        self._prefix.record(page_idx, token_ids, logical_page_idx)


class TaskTable:
    """task_id -> page list and cached-token count."""

    def __init__(self, page_size: int):
        self._page_size = page_size
        self._pages: Dict[str, List[int]] = {}
        self._cached: Dict[str, int] = {}
        self._lock = threading.Lock()

    def set(self, task_id: str, page_table: List[int], cached: int) -> None:
        with self._lock:
            self._pages[task_id] = page_table
            self._cached[task_id] = cached

    def get(self, task_id: str) -> List[int]:
        with self._lock:
            return self._pages.get(task_id, [])

    def get_cached(self, task_id: str) -> int:
        with self._lock:
            return self._cached.get(task_id, 0)

    def pop(self, task_id: str) -> Tuple[List[int], int]:
        with self._lock:
            return self._pages.pop(task_id, []), self._cached.pop(task_id, 0)

    def get_ref(self, task_id: str) -> List[int]:
        with self._lock:
            return self._pages.setdefault(task_id, [])

    def table_tensor(self, task_ids: List[str], device, dtype=torch.long, width: Optional[int] = None) -> Tensor:
        with self._lock:
            rows = [self._pages.get(t, []) for t in task_ids]
        w = max((len(r) for r in rows), default=0) if width is None else width
        return torch.tensor([r + [-1] * (w - len(r)) for r in rows], dtype=dtype).to(device)


class Storage:
    """K/V pages ``[n_layers, n_pages, Hkv, page_size, head_dim]``."""

    def __init__(self, n_layers: int, n_pages: int, page_size: int, n_kv_heads: int, head_dim: int, device,
                 dtype: torch.dtype):
        self.n_layers, self.n_pages, self.page_size = n_layers, n_pages, page_size
        self.n_kv_heads, self.head_dim = n_kv_heads, head_dim
        shape = (n_layers, n_pages, n_kv_heads, page_size, head_dim)
        self.k_cache = torch.zeros(shape, device=device, dtype=dtype)
        self.v_cache = torch.zeros(shape, device=device, dtype=dtype)

    @property
    def native_ok(self) -> bool:
        return self.k_cache.is_cuda and self.k_cache.dtype == torch.bfloat16 and self.head_dim in KERNEL_HEAD_DIMS

    # --------------------------------------------------------------- slot-level primitives
    def write_slots(self, layer_id: int, slots: Tensor, k: Tensor, v: Tensor) -> None:
        """Rows ``k/v [T, >= Hkv*D]`` go to flat slots ``page*page_size + offset`` (-1 skips)."""
        if self.native_ok:
            from astrai_b200.ops._ext import native

            native().paged_kv_write(k, v, slots, self.k_cache[layer_id], self.v_cache[layer_id])
            return
        H, D = self.n_kv_heads, self.head_dim
        ok = slots >= 0
        s = slots[ok].long()
        page, off = s // self.page_size, s % self.page_size
        kk = k[ok][:, : H * D].reshape(-1, H, D).to(self.k_cache.dtype)
        vv = v[ok][:, : H * D].reshape(-1, H, D).to(self.v_cache.dtype)
        heads = torch.arange(H, device=s.device)
        self.k_cache[layer_id][page[:, None], heads[None, :], off[:, None]] = kk
        self.v_cache[layer_id][page[:, None], heads[None, :], off[:, None]] = vv

    def gather_rows(self, layer_id: int, table: Tensor, lens: Tensor, total: int) -> Tuple[Tensor, Tensor]:
        """-> k, v ``[B, total, Hkv, D]`` (zeros past each row's length)."""
        if self.native_ok:
            from astrai_b200.ops._ext import native

            k, v = native().paged_kv_gather(self.k_cache[layer_id], self.v_cache[layer_id],
                                            table.to(torch.int32).contiguous(), lens.to(torch.int32).contiguous(),
                                            int(total))
            return k, v
        B = table.shape[0]
        pos = torch.arange(total, device=table.device)
        raw = pos // self.page_size
        pidx = raw.clamp(max=max(table.shape[1] - 1, 0))
        pages = table.long()[:, pidx] if table.shape[1] else torch.full((B, total), -1, device=table.device)
        valid = (pages >= 0) & (pos[None, :] < lens.long()[:, None]) & (raw < table.shape[1])[None, :]
        p = pages.clamp(min=0)
        off = (pos % self.page_size)[None, :].expand(B, -1)
        k = self.k_cache[layer_id][p, :, off]  # [B, total, H, D]
        v = self.v_cache[layer_id][p, :, off]
        m = valid[:, :, None, None]
        return k.masked_fill(~m, 0), v.masked_fill(~m, 0)

    # --------------------------------------------------------------- reference-shaped API
    def write(self, layer_id: int, page_table: Tensor, start_pos: int, k: Tensor, v: Tensor) -> None:
        """k/v ``[B, S, Hkv, D]`` at positions ``start_pos ..`` of every row."""
        B, S = k.shape[:2]
        if S == 0:
            return
        slots = _slots_uniform(page_table, start_pos, S, self.page_size)
        self.write_slots(layer_id, slots, k.reshape(B * S, -1).contiguous(), v.reshape(B * S, -1).contiguous())

    def gather(self, layer_id: int, page_table: Tensor, total_len: int) -> Tuple[Tensor, Tensor]:
        lens = torch.full((page_table.shape[0],), total_len, dtype=torch.int32, device=page_table.device)
        return self.gather_rows(layer_id, page_table, lens, total_len)


def _slots_uniform(table: Tensor, start: int, S: int, page_size: int) -> Tensor:
    pos = torch.arange(start, start + S, device=table.device)
    pages = table.long()[:, pos // page_size]
    return torch.where(pages >= 0, pages * page_size + pos % page_size, -1).reshape(-1).to(torch.int32)


class CacheView(ABC):
    """What attention layers see of the cache during one forward."""

    @abstractmethod
    def write(self, layer_id: int, k: Tensor, v: Tensor): ...

    @abstractmethod
    def gather(self, layer_id: int) -> Tuple[Tensor, Tensor]: ...

    def attend(self, layer_id: int, q: Tensor, k: Tensor, v: Tensor) -> Tensor:
        """Write the new k/v, then causal attention of q over the cached keys."""
        raise NotImplementedError


class KVCache(ABC):
    """Cache facade used by the scheduler / executor."""

    page_size: int = 64

    @abstractmethod
    def task_alloc(self, task_id: str, prompt_ids: List[int]) -> bool: ...

    @abstractmethod
    def task_free(self, task_id: str): ...

    @abstractmethod
    def task_extend(self, task_id: str, pos: int) -> bool: ...

    @abstractmethod
    def bind_tasks(self, task_ids: List[str], total_len: int, device, write_positions: Optional[Tensor] = None
                   ) -> CacheView: ...

    def task_cached(self, task_id: str) -> int:
        return 0

    def task_record_hashes(self, task_id: str, prompt_ids: List[int], start_logical_page: int = 0): ...


class PageCacheView(CacheView):
    """A batch bound to pages: ``lens[b]`` = keys of row b after this step.

    Built by the caches (``bind_tasks`` / ``bind``); the reference-shaped
    constructor ``PageCacheView(storage, page_table, total_len)`` gives every
    row the same length.
    """

    def __init__(self, storage: Storage, page_table: Tensor, total_len: int = 0, lens: Optional[Tensor] = None,
                 n_new: Optional[int] = None, positions: Optional[Tensor] = None, workspace: Optional[Tensor] = None,
                 splits: Optional[int] = None, uniform_start: Optional[int] = None):
        self._storage = storage
        dev = page_table.device
        self.table = page_table.to(torch.int32).contiguous()
        self.B = self.table.shape[0]
        if lens is None:
            lens = torch.full((self.B,), total_len, dtype=torch.int32, device=dev)
            uniform_start = None  # derived per call from total_len and S
        self.lens = lens.to(torch.int32)
        self._total_len = int(total_len)
        self.uniform_start = uniform_start
        self.n_new = n_new
        self._positions = positions
        self._slots: Dict[int, Tensor] = {}
        self._workspace = workspace
        self._splits = splits

    @property
    def supports_qkv(self) -> bool:
        """True when :meth:`attend_qkv` runs natively (CUDA bf16, head dim 64 or 128)."""
        return self._storage.native_ok

    # ------------------------------------------------------------ geometry
    def positions(self, S: int) -> Tensor:
        """int32 ``[B*S]`` absolute positions of the new tokens."""
        if self._positions is not None and self._positions.numel() == self.B * S:
            return self._positions
        start = self.lens[:, None] - S
        return (start + torch.arange(S, device=self.lens.device, dtype=torch.int32)[None, :]).reshape(-1)

    def slots(self, S: int) -> Tensor:
        if S not in self._slots:
            pos = self.positions(S).view(self.B, S).long()
            ps = self._storage.page_size
            raw = pos // ps
            pidx = raw.clamp(min=0, max=max(self.table.shape[1] - 1, 0))
            pages = self.table.long().gather(1, pidx) if self.table.shape[1] else torch.full_like(pos, -1)
            ok = (pages >= 0) & (pos >= 0) & (raw < self.table.shape[1])  # past the table: not written
            self._slots[S] = torch.where(ok, pages * ps + pos % ps, -1).reshape(-1).to(torch.int32).contiguous()
        return self._slots[S]

    def _start(self, S: int) -> Optional[int]:
        if self.uniform_start is not None:
            return self.uniform_start
        if self.n_new is None and self._total_len:
            return self._total_len - S
        return None

    # ------------------------------------------------------------ reference-shaped API
    def write(self, layer_id: int, k: Tensor, v: Tensor) -> None:
        B, S = k.shape[:2]
        self._storage.write_slots(layer_id, self.slots(S), k.reshape(B * S, -1).contiguous(),
                                  v.reshape(B * S, -1).contiguous())

    def gather(self, layer_id: int) -> Tuple[Tensor, Tensor]:
        total = self._total_len or int(self.lens.max())
        return self._storage.gather_rows(layer_id, self.table, self.lens, total)

    # ------------------------------------------------------------ attention
    def _decode_native(self, layer_id: int, q_rows: Tensor, Hq: int) -> Tensor:
        from astrai_b200.ops._ext import native

        st = self._storage
        C = native()
        if self._splits is None:
            cap = self.table.shape[1] * st.page_size
            self._splits = int(C.decode_splits(self.B, st.n_kv_heads, cap, q_rows.device.index or 0))
        D = st.head_dim
        need = self.B * Hq * self._splits * (D + 2)
        if self._splits > 1 and (self._workspace is None or self._workspace.numel() < need):
            self._workspace = torch.empty(need, device=q_rows.device, dtype=torch.float32)
        out = torch.empty((self.B, Hq * D), device=q_rows.device, dtype=torch.bfloat16)
        C.paged_decode(q_rows, st.k_cache[layer_id], st.v_cache[layer_id], self.table, self.lens, out, Hq,
                       1.0 / math.sqrt(D), self._splits, self._workspace)
        return out

    def attend(self, layer_id: int, q: Tensor, k: Tensor, v: Tensor) -> Tensor:
        """q ``[B,S,Hq,D]``, k/v ``[B,S,Hkv,D]`` (RoPE applied) -> ``[B,S,Hq,D]``."""
        from astrai_b200.ops.attention import attention, attention_reference

        B, S, Hq, D = q.shape
        self.write(layer_id, k, v)
        native = self._storage.native_ok and D == self._storage.head_dim and q.dtype == torch.bfloat16
        if native and S == 1:
            o = self._decode_native(layer_id, q.reshape(B, Hq * D).contiguous(), Hq)
            return o.view(B, 1, Hq, D)
        start = self._start(S)
        if start == 0:
            return attention(q, k, v, causal=True)
        if start is not None:
            kk, vv = self._storage.gather_rows(layer_id, self.table, self.lens, start + S)
            return attention(q, kk, vv, causal=True)
        return self._ragged(layer_id, q, B, S, Hq)  # rows of different lengths

    def attend_qkv(self, layer_id: int, qkv: Tensor, B: int, S: int, Hq: int, Hkv: int, table: Tensor) -> Tensor:
        """Fused path on a ``[B*S, (Hq+2Hkv)*D]`` bf16 buffer (D = 64 or 128): RoPE in place,
        K/V written straight from the buffer, attention -> ``[B*S, Hq*D]``."""
        from astrai_b200.ops.attention import flash_forward
        from astrai_b200.ops.rope import rope_inplace

        D = self._storage.head_dim
        pos = self.positions(S)
        rope_inplace(qkv, 0, Hq + Hkv, D, table, pos, S)
        self._storage.write_slots(layer_id, self.slots(S), qkv[:, Hq * D:(Hq + Hkv) * D],
                                  qkv[:, (Hq + Hkv) * D:])
        if S == 1:
            return self._decode_native(layer_id, qkv, Hq)
        o = torch.empty((B * S, Hq * D), device=qkv.device, dtype=torch.bfloat16)
        lse = torch.empty((B, Hq, S), device=qkv.device, dtype=torch.float32)
        scale = 1.0 / math.sqrt(D)
        start = self._start(S)
        if start == 0:
            flash_forward(qkv, 0, qkv, Hq * D, qkv, (Hq + Hkv) * D, o, lse, B, S, S, Hq, Hkv, D, scale, True, None)
            return o
        if start is None:  # rows of different lengths (RoPE already applied in place)
            q = qkv[:, : Hq * D].reshape(B, S, Hq, D)
            return self._ragged(layer_id, q, B, S, Hq).reshape(B * S, Hq * D)
        total = start + S
        kk, vv = self._storage.gather_rows(layer_id, self.table, self.lens, total)
        flash_forward(qkv, 0, kk.view(B * total, Hkv * D), 0, vv.view(B * total, Hkv * D), 0, o, lse, B, S, total,
                      Hq, Hkv, D, scale, True, None)
        return o

    def _ragged(self, layer_id: int, q: Tensor, B: int, S: int, Hq: int) -> Tensor:
        from astrai_b200.models.components.attention import _dense_attention

        total = int(self.lens.max())
        kk, vv = self._storage.gather_rows(layer_id, self.table, self.lens, total)
        pos = self.positions(S).view(B, S).long()
        keys = torch.arange(total, device=q.device)
        mask = (keys[None, None, :] <= pos[:, :, None])[:, None]
        return _dense_attention(q, kk, vv, mask)


class _TableCache(KVCache):
    """Shared binding logic of both caches."""

    _storage: Storage
    _table: TaskTable

    @property
    def storage(self) -> Storage:
        return self._storage

    def bind(self, task_ids: List[str], lens: Sequence[int], n_new: int, device, uniform_start: Optional[int] = None,
             width: Optional[int] = None) -> PageCacheView:
        """Rows of ``task_ids`` with ``lens[b]`` keys after appending ``n_new`` tokens."""
        table = self._table.table_tensor(task_ids, "cpu", torch.int32, width)
        ln = torch.tensor(list(lens), dtype=torch.int32)
        return PageCacheView(self._storage, table.to(device, non_blocking=True), lens=ln.to(device, non_blocking=True),
                             n_new=n_new, uniform_start=uniform_start)

    def bind_tasks(self, task_ids: List[str], total_len: int, device, write_positions: Optional[Tensor] = None
                   ) -> PageCacheView:
        if write_positions is not None:  # decode: per-row positions, one new token
            lens = [int(p) + 1 for p in write_positions.reshape(-1).tolist()]
            return self.bind(task_ids, lens, 1, device)
        return PageCacheView(self._storage, self._table.table_tensor(task_ids, device, torch.int32), total_len)


class PageCache(_TableCache):
    """Paged KV cache with prefix sharing across tasks."""

    def __init__(self, n_layers: int, n_pages: int, page_size: int, n_kv_heads: int, head_dim: int, device,
                 dtype: torch.dtype):
        self.page_size = page_size
        self._pool = PagePool(Allocator(n_pages), PrefixCache(page_size))
        self._table = TaskTable(page_size)
        self._storage = Storage(n_layers, n_pages, page_size, n_kv_heads, head_dim, device, dtype)

    @property
    def pool(self) -> PagePool:
        return self._pool

    def task_alloc(self, task_id: str, prompt_ids: List[int]) -> bool:
        # never hit the page holding the last prompt token: it is recomputed
        hits = self._pool.lookup(prompt_ids, max_pages=(len(prompt_ids) - 1) // self.page_size)
        for p in hits:
            self._pool.inc_ref(p)
        cached = len(hits) * self.page_size
        n_new = -(-(len(prompt_ids) - cached) // self.page_size)
        new_pages: List[int] = []
        for _ in range(max(n_new, 0)):
            p = self._pool.alloc()
            if p < 0:
                for q in hits + new_pages:
                    self._pool.free(q)
                return False
            new_pages.append(p)
        self._table.set(task_id, hits + new_pages, cached)
        return True

    def task_free(self, task_id: str) -> None:
        pages, _ = self._table.pop(task_id)
        for p in pages:
            self._pool.free(p)

    def task_extend(self, task_id: str, pos: int) -> bool:
        pages = self._table.get_ref(task_id)
        need = pos // self.page_size + 1
        while len(pages) < need:
            p = self._pool.alloc()
            if p < 0:
                return False
            pages.append(p)
        return True

    def task_cached(self, task_id: str) -> int:
        return self._table.get_cached(task_id)

    def task_record_hashes(self, task_id: str, prompt_ids: List[int], start_logical_page: int = 0) -> None:
        pages = self._table.get(task_id)
        full = len(prompt_ids) // self.page_size
        hashes = _page_hashes(prompt_ids, full, self.page_size)
        for i in range(start_logical_page, min(full, len(pages))):
            self._pool.prefix.record_hash(pages[i], hashes[i])


class ContiguousCacheView(PageCacheView):
    """Per-slot view (a slot is one page of ``max_seq_len`` keys)."""


class ContiguousCache(_TableCache):
    """One slot of ``max_seq_len`` keys per running task (no sharing)."""

    def __init__(self, n_layers: int, max_batch_size: int, max_seq_len: int, n_kv_heads: int, head_dim: int, device,
                 dtype: torch.dtype):
        self.max_seq_len = max_seq_len
        # a slot holds max_seq_len keys, rounded up to the 128-key tile of the tensor-core decode kernel
        # (its TMA boxes never straddle two slots); the capacity checks still use max_seq_len
        self.page_size = (max_seq_len + 127) // 128 * 128
        self._storage = Storage(n_layers, max_batch_size, self.page_size, n_kv_heads, head_dim, device, dtype)
        self._table = TaskTable(self.page_size)
        self._free_slots = list(range(max_batch_size))
        self._lock = threading.Lock()

    @property
    def k(self) -> Tensor:
        return self._storage.k_cache

    @property
    def v(self) -> Tensor:
        return self._storage.v_cache

    def task_alloc(self, task_id: str, prompt_ids: List[int]) -> bool:
        with self._lock:
            if not self._free_slots or len(prompt_ids) > self.max_seq_len:
                return False
            slot = self._free_slots.pop(0)
        self._table.set(task_id, [slot], 0)
        return True

    def task_free(self, task_id: str) -> None:
        pages, _ = self._table.pop(task_id)
        with self._lock:
            self._free_slots.extend(pages)

    def task_extend(self, task_id: str, pos: int) -> bool:
        return pos < self.max_seq_len and bool(self._table.get(task_id))

    def task_cached(self, task_id: str) -> int:
        return 0
