"""Logical-shadow checker on the device (diagnostic bitwise KV validation).

Mirrors LogicalShadow of adaptive_sparse/logical_shadow.py:14-140: the same
constructor, attributes (``layers``, ``counts``, ``dirty``,
``migration_counts``), methods (``reset``, ``write``, ``check``,
``check_complete``, ``publish``), errors and returned tensors.  The torch
bodies become four kernels of libekv_b200.so (``ekv_shadow_write``,
``ekv_shadow_reset``, ``ekv_shadow_check``, ``ekv_shadow_check_complete``), so
a correctness run compares every selected and every migrated row at HBM speed
and its counters stay on the device until ``publish``.

The SGLang hooks that feed it (``install_logical_shadow``) patch a
third-party engine and are not part of this package.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from ._lib import SHADOW_MAX_LAYERS, call, index_esize, stream_handle, u64_array

_TWO_BYTE = (torch.bfloat16, torch.float16, torch.int16)


def _slot_rows(tensor: torch.Tensor, name: str) -> tuple[int, int]:
    """(row bytes, slot stride in bytes) of a [slots, ...] buffer with contiguous rows."""
    if tensor.dtype not in _TWO_BYTE:
        raise ValueError(f"{name} must hold 2-byte (bf16) rows")
    if tensor.dim() < 1 or (tensor.dim() > 1 and not tensor[0].is_contiguous()):
        raise ValueError(f"{name} rows must be contiguous")
    elements = 1
    for size in tensor.shape[1:]:
        elements *= size
    return elements * tensor.element_size(), tensor.stride(0) * tensor.element_size()


def _index(tensor: torch.Tensor, device: torch.device) -> torch.Tensor:
    if tensor.device != device:
        tensor = tensor.to(device)
    if tensor.dtype not in (torch.int32, torch.int64):
        tensor = tensor.to(torch.int64)
    return tensor


def _flat_index(tensor, device) -> torch.Tensor:
    tensor = torch.as_tensor(tensor, device=device)
    return _index(tensor, device).reshape(-1).contiguous()


class LogicalShadow:
    def __init__(self, capacity, device):
        self.capacity = capacity
        self.device = device
        self.layers = {}
        self.counts = torch.zeros(7, device=device, dtype=torch.int64)
        self.dirty = False
        self.migration_counts = dict.fromkeys((
            "migration_checked_tokens", "migration_checked_bytes",
            "migration_invalid_tokens", "migration_mismatched_tokens",
        ), 0)

    # ------------------------------------------------------------------ producers

    def reset(self, locations):
        """Forget the slots in ``locations`` on every layer (logical_shadow.py:26-28)."""
        if not self.layers:
            return
        device = torch.device(self.device)
        loc = _flat_index(locations, device)
        if not loc.numel():
            return
        flags = [valid for _, _, valid in self.layers.values()]
        for start in range(0, len(flags), SHADOW_MAX_LAYERS):
            group = flags[start:start + SHADOW_MAX_LAYERS]
            call("ekv_shadow_reset", u64_array(f.data_ptr() for f in group), len(group), self.capacity,
                 loc.data_ptr(), index_esize(loc, "locations"), loc.numel(), device.index, stream_handle(device))

    def write(self, layer, locations, key, value, scales):
        """Record a producer write (logical_shadow.py:30-43)."""
        if (key.dtype != torch.bfloat16 or value.dtype != torch.bfloat16
                or any(scale not in (None, 1.0) for scale in scales)):
            raise RuntimeError("Logical shadow requires unit-scale BF16 producers")
        if layer not in self.layers:
            self.layers[layer] = (
                key.new_empty((self.capacity, *key.shape[1:])),
                value.new_empty((self.capacity, *value.shape[1:])),
                torch.zeros(self.capacity, device=self.device, dtype=torch.bool),
            )
        k, v, valid = self.layers[layer]
        device = k.device
        loc = _flat_index(locations, device)
        if key.shape[1:] != k.shape[1:] or value.shape[1:] != v.shape[1:]:
            raise ValueError("producer rows do not match the shadow's row shape")
        if key.shape[0] != loc.numel() or value.shape[0] != loc.numel():
            raise ValueError("one key and one value row per location")
        key = key if key.shape[0] == 0 or key[0].is_contiguous() else key.contiguous()
        value = value if value.shape[0] == 0 or value[0].is_contiguous() else value.contiguous()
        k_bytes, k_stride = _slot_rows(k, "shadow K")
        v_bytes, v_stride = _slot_rows(v, "shadow V")
        _, key_stride = _slot_rows(key, "key")
        _, value_stride = _slot_rows(value, "value")
        call("ekv_shadow_write", k.data_ptr(), v.data_ptr(), valid.data_ptr(), self.capacity, k_stride, v_stride,
             key.data_ptr(), value.data_ptr(), key_stride, value_stride, k_bytes, v_bytes,
             loc.data_ptr(), index_esize(loc, "locations"), loc.numel(), device.index, stream_handle(device))

    # ------------------------------------------------------------------ checks

    def check(self, layer, k_cache, v_cache, table, lengths, rows, block_size,
              blocks, physical, live_pages, page_size):
        """One decode step of one layer (logical_shadow.py:45-86).

        Returns ``(clean_blocks, physical_out)``: the Top-K ids with everything
        after each row's valid prefix set to -1, and the physical slots (int32
        ``[1, B, K * block_size]``) with unbacked selected slots set to 0.  The
        seven counters accumulate in ``self.counts`` on the device.
        """
        if layer not in self.layers or blocks.shape[0] != 1:
            raise RuntimeError("Logical shadow requires one KV head and recorded producer writes")
        k, v, initialized = self.layers[layer]
        device = k.device
        if blocks.dim() != 3 or blocks.dtype not in (torch.int32, torch.int64):
            raise ValueError("blocks must be an int32 / int64 tensor [1, batch, blocks]")
        batch, n_blocks = blocks.shape[1], blocks.shape[2]
        if k_cache.shape[1:] != k.shape[1:] or v_cache.shape[1:] != v.shape[1:]:
            raise ValueError("cache rows and shadow rows differ in shape")
        k_bytes, k_cache_stride = _slot_rows(k_cache, "k_cache")
        v_bytes, v_cache_stride = _slot_rows(v_cache, "v_cache")
        _, k_shadow_stride = _slot_rows(k, "shadow K")
        _, v_shadow_stride = _slot_rows(v, "shadow V")
        blocks = blocks.to(device)
        lengths_t = _index(lengths.reshape(-1), device)
        rows_t = _index(rows.reshape(-1), device)
        table_t = _index(table, device)
        width = n_blocks * block_size
        phys_ptr, phys_row, phys_col = None, 0, 0
        if physical is not None:
            if physical.dtype != torch.int32 or physical.shape != (1, batch, width):
                raise ValueError("physical must be int32 [1, batch, blocks * block_size]")
            physical = physical.to(device)
            phys_ptr, phys_row, phys_col = physical.data_ptr(), physical.stride(1), physical.stride(2)
        live_ptr, live_len = None, 0
        if live_pages is not None:
            live = live_pages.to(device).reshape(-1).contiguous()
            live = live.view(torch.uint8) if live.dtype == torch.bool else live.to(torch.uint8)
            live_ptr, live_len = live.data_ptr(), live.numel()
        clean = torch.empty((1, batch, n_blocks), dtype=blocks.dtype, device=device)
        physical_out = torch.empty((1, batch, width), dtype=torch.int32, device=device)
        call("ekv_shadow_check",
             blocks.data_ptr(), blocks.element_size(), batch, n_blocks, blocks.stride(1), blocks.stride(2),
             lengths_t.data_ptr(), index_esize(lengths_t, "lengths"), lengths_t.stride(0),
             rows_t.data_ptr(), index_esize(rows_t, "rows"), rows_t.stride(0),
             table_t.data_ptr(), index_esize(table_t, "table"), table_t.shape[1], table_t.stride(0),
             table_t.stride(1), phys_ptr, phys_row, phys_col, live_ptr, live_len,
             k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0], k_cache_stride, v_cache_stride,
             k.data_ptr(), v.data_ptr(), initialized.data_ptr(), self.capacity, k_shadow_stride, v_shadow_stride,
             k_bytes, v_bytes, block_size, page_size, clean.data_ptr(), physical_out.data_ptr(),
             self.counts.data_ptr(), device.index, stream_handle(device))
        self.dirty = True
        return clean, physical_out

    def check_complete(self, pool, logical, physical, boundary):
        """Compare every committed token in the migrated sparse main layers
        (logical_shadow.py:88-123)."""
        if logical.ndim != 1 or physical.shape != logical.shape or not logical.numel():
            raise ValueError("Invalid migration shadow slot vectors")
        page = pool.page_size
        layers = list(range(pool.start_layer, pool.end_layer))
        for layer in layers:
            if layer not in self.layers:
                raise RuntimeError(f"Missing migration shadow writes for layer {layer}")
        device = torch.device(self.device)
        # The live-page mask: a scatter, so the page set needs no sorting.
        pages = pool.adaptive_vmm.pages
        live_host = np.zeros(pool.size // page + 1, dtype=np.uint8)
        live_host[np.fromiter(pages, dtype=np.int64, count=len(pages))] = 1
        live = torch.from_numpy(live_host).to(device)
        counts = torch.zeros(4, device=device, dtype=torch.int64)
        self.launch_complete(pool, layers, _index(logical, device), _index(physical, device), live, counts)
        report = dict(zip(self.migration_counts, counts.tolist(), strict=True))
        for name, count in report.items():
            self.migration_counts[name] += count
        self.dirty = True
        if report["migration_invalid_tokens"] or report["migration_mismatched_tokens"]:
            raise RuntimeError(f"Logical KV migration shadow mismatch at {boundary}: {report}")

    def launch_complete(self, pool, layers, logical, physical, live, counts):
        """The device part of ``check_complete``: ADD the four migration counters of
        ``layers`` to ``counts`` (int64 [4] on the device) without synchronizing.
        ``live`` is the uint8 live-page mask [pool.size // page_size + 1]."""
        page = pool.page_size
        device = torch.device(self.device)
        groups: dict[tuple, list] = {}
        for layer in layers:
            key, value, initialized = self.layers[layer]
            pool_k, pool_v = pool.get_key_buffer(layer), pool.get_value_buffer(layer)
            if pool_k.shape[0] < pool.size + page or pool_v.shape[0] < pool.size + page:
                raise ValueError("pool buffers must hold size + page_size slots")
            if pool_k.shape[1:] != key.shape[1:] or pool_v.shape[1:] != value.shape[1:]:
                raise ValueError("pool rows and shadow rows differ in shape")
            kb, pks = _slot_rows(pool_k, "pool K")
            vb, pvs = _slot_rows(pool_v, "pool V")
            _, sks = _slot_rows(key, "shadow K")
            _, svs = _slot_rows(value, "shadow V")
            groups.setdefault((kb, vb, pks, pvs, sks, svs), []).append(
                (pool_k.data_ptr(), pool_v.data_ptr(), key.data_ptr(), value.data_ptr(), initialized.data_ptr()))
        for (kb, vb, pks, pvs, sks, svs), members in groups.items():
            for start in range(0, len(members), SHADOW_MAX_LAYERS):
                part = members[start:start + SHADOW_MAX_LAYERS]
                columns = list(zip(*part))
                call("ekv_shadow_check_complete",
                     logical.data_ptr(), index_esize(logical, "logical"),
                     physical.data_ptr(), index_esize(physical, "physical"), logical.numel(),
                     page, pool.size, self.capacity, live.data_ptr(), live.numel(),
                     *(u64_array(c) for c in columns), len(part), pks, pvs, sks, svs, kb, vb,
                     counts.data_ptr(), device.index, stream_handle(device))

    def publish(self, directory, rank):
        """Write shadow-tp-<rank>.json and raise on any mismatch (logical_shadow.py:125-140)."""
        if not self.dirty:
            return
        keys = ("checked_tokens", "checked_bytes", "uninitialized_logical_tokens",
                "invalid_physical_tokens", "mismatched_tokens", "checked_calls",
                "malformed_topk_blocks")
        stats = dict(zip(keys, self.counts.tolist(), strict=True))
        stats.update(self.migration_counts)
        stats.update(tp_rank=rank, logical_capacity=self.capacity, boundary="scheduler_idle")
        path = Path(directory) / f"shadow-tp-{rank}.json"
        tmp = path.with_suffix(".tmp")
        tmp.write_text(json.dumps(stats, indent=2) + "\n", encoding="utf-8")
        tmp.replace(path)
        self.dirty = False
        if any(stats[key] for key in (*keys[2:5], keys[6])):
            raise RuntimeError(f"Logical KV shadow mismatch: {stats}")
