"""Demote / promote transactions for long host-backed requests (R5).

Same functions, arguments, state machine (prepared -> committing -> committed |
aborted) and error types as the reference's adaptive_sparse/migration.py:27-288,
so the scheduler hook drives them unchanged.  The bytes move through the
coordinator's host pool; with ``host_pool.PinnedHostKVPool`` installed as
``coordinator.mem_pool_host`` every row copy is one launch of the sm_100a
pack/unpack kernel over all planes instead of per-layer library calls.

The scheduler must pause decode and agree on prepare success across ranks
before committing; a commit failure is fail-stop across the TP group.
"""

from __future__ import annotations

import os
from collections import Counter
from dataclasses import dataclass

from .profile_ranges import profile_range


@dataclass
class PreparedDemotion:
    coordinator: object
    request: object
    row: int
    logical: object
    physical: object
    committed_len: int
    retained_rows: tuple
    released_rows: tuple
    status: str = "prepared"


@dataclass
class PreparedPromotion:
    coordinator: object
    request: object
    row: int
    logical: object
    destination: object
    backed_before: int
    status: str = "prepared"


def plan_demote_pages(tracker, page_ids, keep_pages):
    """Split ``page_ids`` into (kept-as-hot-buffer, released) pages.

    Default: keep the first ``keep_pages`` pages.  With
    ``EKV_CHUNK_AWARE_RETENTION=1`` pages are kept greedily so that as few
    request-exclusive chunks as possible stay referenced: each step keeps the
    page adding the fewest new exclusive chunks, preferring a chunk signature
    that more remaining pages share, then the lowest page id
    (adaptive_sparse/migration.py:27-54).
    """
    pages = tuple(page_ids)
    if not 0 < keep_pages <= len(pages) or len(set(pages)) != len(pages):
        raise ValueError("Invalid demotion page ownership")
    if os.environ.get("EKV_CHUNK_AWARE_RETENTION") != "1":
        return pages[:keep_pages], pages[keep_pages:]
    if tracker is None:
        raise RuntimeError("Chunk-aware retention requires a physical page tracker")
    chunks_of = {page: tracker.chunks(page) for page in pages}
    holders = Counter(chunk for chunks in chunks_of.values() for chunk in chunks)
    # Chunks every one of whose references is a page of this request.
    exclusive = {chunk for chunk, n in holders.items() if n == tracker.refs.get(chunk)}
    kept_chunks = set()
    left = set(pages)
    kept = []
    for _ in range(keep_pages):
        added = {page: frozenset((chunks_of[page] & exclusive) - kept_chunks) for page in left}
        popularity = Counter(added.values())
        choice = min(left, key=lambda page: (len(added[page]), -popularity[added[page]], page))
        kept.append(choice)
        kept_chunks.update(chunks_of[choice] & exclusive)
        left.remove(choice)
    return tuple(kept), tuple(page for page in pages if page in left)


def _release_host(coordinator, row):
    host_pool = coordinator.mem_pool_host
    indices = host_pool.allocated_host_indices(
        coordinator.req_to_host_pool, row, coordinator.req_to_host_pool_allocated_len[row])
    if indices.numel():
        host_pool.free(indices)
    coordinator.req_to_host_pool[row].fill_(-1)
    coordinator.req_to_host_pool_allocated_len[row] = 0


@profile_range("hisparse/demotion/prepare")
def prepare_demote(coordinator, req, synchronize):
    """Copy a resident request's committed K/V to the host without changing ownership."""
    if not coordinator.is_m3_hisparse or coordinator.spec_swap.enabled:
        raise RuntimeError("Demotion requires native M3 HiSparse without speculation")
    kv = req.kv
    row, length = kv.req_pool_idx, kv.kv_committed_len
    if (row is None or req.hisparse_staging or length != kv.kv_allocated_len
            or length < coordinator.padded_buffer_size):
        raise ValueError("Demotion requires a fully committed long resident request")
    if (int(coordinator.req_device_buffer_size[row])
            or int(coordinator.req_to_host_pool_allocated_len[row])):
        raise RuntimeError("Resident request unexpectedly owns HiSparse cache state")
    device_pool = coordinator.mem_pool_device
    page_size = device_pool.page_size
    if coordinator.padded_buffer_size % page_size:
        raise RuntimeError("Hot buffer must be page-aligned")
    logical = coordinator.req_to_token_pool.req_to_token[row, :length].clone()
    physical = device_pool.translate_loc_from_full_to_hisparse_device(logical)
    if not bool((physical > 0).all()):
        raise RuntimeError("Resident request has missing physical locations")
    starts = physical[::page_size].tolist()
    if any(slot % page_size for slot in starts):
        raise RuntimeError("Resident request page starts are misaligned")
    page_ids = [slot // page_size for slot in starts]
    if len(page_ids) != len(set(page_ids)):
        raise RuntimeError("Resident request reuses a physical page")
    tracker = getattr(device_pool, "adaptive_vmm", None)
    kept, released = plan_demote_pages(tracker, page_ids, coordinator.padded_buffer_size // page_size)
    position = {page: index for index, page in enumerate(page_ids)}
    retained_rows = tuple(position[page] for page in kept)
    released_rows = tuple(position[page] for page in released)
    coordinator.wait_for_pending_backup()
    synchronize()
    shadow = getattr(coordinator.token_to_kv_pool_allocator._kvcache, "_ekv_shadow", None)
    if shadow is not None:
        shadow.check_complete(device_pool, logical, physical, "demote_source")
    try:
        host = coordinator.mem_pool_host.alloc_paged_token_slots(
            coordinator.req_to_host_pool, coordinator.req_to_host_pool_allocated_len, row, 0, length)
        coordinator.mem_pool_host.backup_from_device_all_layer(device_pool, host, physical,
                                                               io_backend="kernel")
        synchronize()
    except Exception:
        # A failed synchronize may leave device work referencing the host rows;
        # the fail-stop path owns them then.
        synchronize()
        _release_host(coordinator, row)
        raise
    return PreparedDemotion(coordinator, req, row, logical, physical, length,
                            retained_rows, released_rows)


def abort_demote(prepared):
    """Undo a prepared demotion after the ranks reject it."""
    if prepared.status != "prepared":
        raise RuntimeError("Only a prepared demotion can be aborted")
    _release_host(prepared.coordinator, prepared.row)
    prepared.status = "aborted"


@profile_range("hisparse/demotion/commit")
def commit_demote(prepared, publish_host_backed, synchronize, trim_quiescent=None):
    """Hand the kept pages to the fixed hot buffer and free the rest.

    ``publish_host_backed`` removes the row from resident dispatch; scheduling
    stays paused until every TP rank confirms.
    """
    if prepared.status != "prepared":
        raise RuntimeError("Demotion has already been resolved")
    prepared.status = "committing"
    import torch

    coordinator = prepared.coordinator
    row = prepared.row
    capacity = coordinator.padded_buffer_size
    physical = prepared.physical
    page_size = coordinator.mem_pool_device.page_size
    starts = physical[::page_size]
    kept_rows = torch.tensor(prepared.retained_rows, device=physical.device, dtype=torch.long)
    kept = (starts[kept_rows, None] + torch.arange(page_size, device=physical.device)).flatten()
    kept = kept.to(dtype=coordinator.req_to_device_buffer.dtype)
    coordinator.req_to_device_buffer[row, :capacity] = kept
    coordinator.req_device_buffer_size[row] = capacity
    # The host image just written is authoritative: every lookup starts as a miss.
    coordinator.req_device_buffer_tokens[:, row, :].fill_(-1)
    coordinator.req_device_buffer_token_locs[:, row, :capacity] = kept
    coordinator.lru_slots[:, row, :].copy_(coordinator._lru_init)
    coordinator.spec_swap.reset(row)
    coordinator._skip_first_backup[row] = True
    remove_source = getattr(coordinator, "_ekv_remove_demoted_source", None)
    if remove_source is not None:
        remove_source(prepared.request)
    mapping = coordinator.mem_pool_device.full_to_hisparse_device_index_mapping
    mapping[prepared.logical] = 0
    synchronize()
    released = torch.tensor(prepared.released_rows, device=physical.device, dtype=torch.long)
    coordinator.token_to_kv_pool_allocator.free_hisparse_indices(starts[released])
    synchronize()
    released_bytes = trim_quiescent() if trim_quiescent is not None else 0
    publish_host_backed(row)
    prepared.status = "committed"
    return released_bytes


@profile_range("hisparse/promotion/prepare")
def prepare_promote(coordinator, req, synchronize):
    """Copy host-backed history into fresh physical pages without publishing it."""
    if (not coordinator.is_m3_hisparse or coordinator.spec_swap.enabled
            or coordinator.compress_ratio != 1):
        raise RuntimeError("Promotion requires native M3 HiSparse without speculation")
    kv = req.kv
    row, length = kv.req_pool_idx, kv.kv_committed_len
    if (row is None or req.hisparse_staging or length != kv.kv_allocated_len
            or length <= coordinator.device_buffer_size):
        raise ValueError("Promotion requires a fully committed long host-backed request")
    pool = coordinator.mem_pool_device
    page = pool.page_size
    tracker = getattr(pool, "adaptive_vmm", None)
    if tracker is None:
        raise RuntimeError("Promotion requires the tracked MiniMax VMM main pool")
    if int(coordinator.req_device_buffer_size[row]) != coordinator.padded_buffer_size:
        raise RuntimeError("Unexpected source hot-buffer capacity")
    coordinator.wait_for_pending_backup()
    synchronize()
    logical = coordinator.req_to_token_pool.req_to_token[row, :length].clone()
    host_authoritative = bool(coordinator._skip_first_backup[row])
    host_len = length if host_authoritative else length - 1
    host = coordinator.req_to_host_pool[row, :host_len]
    if (int(coordinator.req_to_host_pool_allocated_len[row]) < host_len
            or not bool((host >= 0).all())):
        raise RuntimeError("Promotion source is missing committed host KV")
    latest = None
    if not host_authoritative:
        latest = coordinator.req_to_device_buffer[row, coordinator.device_buffer_size:][:1]
        if not bool((latest > 0).all()):
            raise RuntimeError("Promotion source is missing the latest device token")
    allocator = coordinator.token_to_kv_pool_allocator
    backed_before = tracker.backing.backed_bytes
    destination = allocator.hisparse_attn_allocator.alloc(-(-length // page) * page)
    if destination is None:
        raise MemoryError("No physical pages available for promotion")
    try:
        for layer in range(pool.start_layer, pool.end_layer):
            coordinator.mem_pool_host.load_to_device_per_layer(
                pool, host, destination[:host_len], layer, io_backend="kernel")
            if latest is not None:
                for buffer in (pool.get_key_buffer(layer), pool.get_value_buffer(layer)):
                    buffer[destination[host_len:host_len + 1]] = buffer[latest]
        synchronize()
        shadow = getattr(allocator._kvcache, "_ekv_shadow", None)
        if shadow is not None:
            shadow.check_complete(pool, logical, destination[:length], "promote_destination")
    except Exception:
        synchronize()
        allocator.free_hisparse_indices(destination)
        tracker.trim_quiescent()
        raise
    return PreparedPromotion(coordinator, req, row, logical, destination, backed_before)


def abort_promote(prepared):
    """Release only the new destination after a rejected prepare vote."""
    if prepared.status != "prepared":
        raise RuntimeError("Only a prepared promotion can be aborted")
    coordinator = prepared.coordinator
    coordinator.token_to_kv_pool_allocator.free_hisparse_indices(prepared.destination)
    coordinator.mem_pool_device.adaptive_vmm.trim_quiescent()
    prepared.status = "aborted"


@profile_range("hisparse/promotion/commit")
def commit_promote(prepared, publish_gpu_resident, synchronize):
    """Release the host-backed source and publish the prepopulated resident mapping."""
    if prepared.status != "prepared":
        raise RuntimeError("Promotion has already been resolved")
    prepared.status = "committing"
    coordinator = prepared.coordinator
    pool = coordinator.mem_pool_device
    # Source cleanup drops host and hot-buffer ownership and old mappings; the
    # residency hook keeps it apart from request completion.
    cleanup = getattr(coordinator, "_ekv_cleanup_promotion_source", None)
    if cleanup is None:
        coordinator.request_finished(prepared.request)
    else:
        cleanup(prepared.request)
    pool.full_to_hisparse_device_index_mapping[prepared.logical] = (
        prepared.destination[:len(prepared.logical)])
    synchronize()
    tracker = pool.adaptive_vmm
    tracker.trim_quiescent()
    publish_gpu_resident(prepared.row)
    register_source = getattr(coordinator, "_ekv_register_promoted_source", None)
    if register_source is not None:
        register_source(prepared.request)
    prepared.status = "committed"
    return max(0, tracker.backing.backed_bytes - prepared.backed_before)
