"""Demote / promote transactions for long host-backed requests (R5).

Public surface of the reference's adaptive_sparse/migration.py:27-288, which the
SGLang scheduler hook calls unchanged: ``plan_demote_pages``,
``prepare_demote`` / ``abort_demote`` / ``commit_demote``, ``prepare_promote``
/ ``abort_promote`` / ``commit_promote``, the ``PreparedDemotion`` /
``PreparedPromotion`` records, the status machine ``prepared -> committing ->
committed | aborted``, the exception types and messages, and the order in
which the coordinator's state is changed (that order is what the other TP
ranks and the scheduler observe).  The implementation is this build's:

* prepare-time validation of the physical locations (all mapped, page starts
  aligned, no page reused) is one device computation and one host read, not a
  device sync per check plus a Python list of every page start;
* the chunk-aware retention planner keeps remaining pages grouped by the set
  of exclusive chunks they would still pin, and updates only the groups the
  last choice touched, instead of recomputing every page's marginal set each
  step (same choices, same tie-breaks);
* promotion restores every layer's K and V in one call when the host pool
  offers ``load_to_device_all_layer`` (``host_pool.PinnedHostKVPool`` does: one
  staged copy-engine transfer over all planes), and copies the newest token's
  rows of all planes in two launches, instead of a loop of per-layer copies
  and 2 x layers indexed assignments.

The scheduler must pause decode and agree on prepare success across ranks
before committing; a commit failure is fail-stop across the TP group.
"""

from __future__ import annotations

import bisect
import os
from collections import Counter, defaultdict
from dataclasses import dataclass

from .profile_ranges import profile_range

_PREPARED, _COMMITTING, _COMMITTED, _ABORTED = "prepared", "committing", "committed", "aborted"


class _Transaction:
    """Status machine shared by both records."""

    _noun = ""

    def _enter_commit(self):
        if self.status != _PREPARED:
            raise RuntimeError(f"{self._noun} has already been resolved")
        self.status = _COMMITTING

    def _check_abortable(self):
        if self.status != _PREPARED:
            raise RuntimeError(f"Only a prepared {self._noun.lower()} can be aborted")


@dataclass
class PreparedDemotion(_Transaction):
    coordinator: object
    request: object
    row: int
    logical: object
    physical: object
    committed_len: int
    retained_rows: tuple
    released_rows: tuple
    status: str = _PREPARED
    _noun = "Demotion"


@dataclass
class PreparedPromotion(_Transaction):
    coordinator: object
    request: object
    row: int
    logical: object
    destination: object
    backed_before: int
    status: str = _PREPARED
    _noun = "Promotion"


# --------------------------------------------------------------------------- planning

class _RetentionGroups:
    """Remaining pages grouped by the exclusive chunks keeping each would still pin.

    ``sig[p]`` is page p's exclusive chunks not yet protected.  Pages with the
    same signature form a group (kept as a sorted list); ``holders[c]`` lists the
    remaining pages whose signature contains chunk c, so protecting chunks
    re-files only those pages.
    """

    def __init__(self, exclusive_of):
        self.sig = dict(exclusive_of)
        self.groups = defaultdict(list)
        self.holders = defaultdict(set)
        for page in sorted(self.sig):
            self.groups[self.sig[page]].append(page)
            for chunk in self.sig[page]:
                self.holders[chunk].add(page)

    def best(self):
        """The page the greedy rule keeps next: fewest newly pinned chunks, then
        the signature most remaining pages share, then the lowest page id."""
        sig, pages = min(self.groups.items(), key=lambda item: (len(item[0]), -len(item[1]), item[1][0]))
        return pages[0]

    def take(self, page):
        """Keep ``page``: drop it and protect its chunks for the pages left."""
        sig = self.sig.pop(page)
        self._unfile(page, sig)
        moved = set()
        for chunk in sig:
            moved |= self.holders.pop(chunk, set())
        for other in sorted(moved):
            old = self.sig[other]
            new = old - sig
            self._unfile(other, old)
            self.sig[other] = new
            bisect.insort(self.groups[new], other)
            for chunk in new:
                self.holders[chunk].add(other)

    def _unfile(self, page, sig):
        group = self.groups[sig]
        del group[bisect.bisect_left(group, page)]
        if not group:
            del self.groups[sig]
        for chunk in sig:
            holders = self.holders.get(chunk)
            if holders is not None:
                holders.discard(page)


def plan_demote_pages(tracker, page_ids, keep_pages):
    """Split ``page_ids`` into (kept as the hot buffer, released) pages.

    Default: keep the first ``keep_pages`` pages.  With
    ``EKV_CHUNK_AWARE_RETENTION=1``: keep, one page at a time, the page whose
    exclusive chunks (chunks no other owner references) add the fewest chunks
    to those already pinned, preferring a signature more remaining pages share,
    then the lowest page id -- the rule of adaptive_sparse/migration.py:27-54.
    """
    pages = tuple(page_ids)
    if not 0 < keep_pages <= len(pages) or len(set(pages)) != len(pages):
        raise ValueError("Invalid demotion page ownership")
    if os.environ.get("EKV_CHUNK_AWARE_RETENTION") != "1":
        return pages[:keep_pages], pages[keep_pages:]
    if tracker is None:
        raise RuntimeError("Chunk-aware retention requires a physical page tracker")
    chunks_of = {page: tracker.chunks(page) for page in pages}
    owned_here = Counter(chunk for chunks in chunks_of.values() for chunk in chunks)
    refs = tracker.refs
    exclusive = {chunk for chunk, n in owned_here.items() if n == refs.get(chunk)}
    groups = _RetentionGroups({page: frozenset(chunks & exclusive) for page, chunks in chunks_of.items()})
    kept = []
    for _ in range(keep_pages):
        page = groups.best()
        groups.take(page)
        kept.append(page)
    released = tuple(page for page in pages if page in groups.sig)
    return tuple(kept), released


# --------------------------------------------------------------------------- helpers

def _release_host(coordinator, row):
    host_pool = coordinator.mem_pool_host
    indices = host_pool.allocated_host_indices(
        coordinator.req_to_host_pool, row, coordinator.req_to_host_pool_allocated_len[row])
    if indices.numel():
        host_pool.free(indices)
    coordinator.req_to_host_pool[row].fill_(-1)
    coordinator.req_to_host_pool_allocated_len[row] = 0


def _physical_pages(physical, page_size):
    """Page ids of a request's physical slots, validated in one device pass.

    Returns the page ids (Python ints, in token order) or raises the first of
    the reference's three errors that applies: a slot that is not mapped
    (<= 0), a page start off the page grid, a page used twice.
    """
    import torch

    starts = physical[::page_size]
    ids = torch.div(starts, page_size, rounding_mode="floor")
    order = torch.sort(ids).values
    verdict = torch.stack([(physical <= 0).any(), (starts % page_size != 0).any(),
                           (order[1:] == order[:-1]).any()]).to(ids.dtype)
    host = torch.cat([verdict, ids]).cpu().tolist()  # the one device -> host read
    missing, misaligned, reused = host[:3]
    if missing:
        raise RuntimeError("Resident request has missing physical locations")
    if misaligned:
        raise RuntimeError("Resident request page starts are misaligned")
    if reused:
        raise RuntimeError("Resident request reuses a physical page")
    return host[3:]


def _page_slots(starts, rows, page_size):
    """Every token slot of the pages ``starts[rows]`` (page order kept)."""
    import torch

    pick = torch.as_tensor(rows, device=starts.device, dtype=torch.long)
    return (starts[pick, None] + torch.arange(page_size, device=starts.device)).flatten()


def _install_hot_buffer(coordinator, row, slots):
    """Hand ``slots`` to the request's fixed hot buffer, every lookup starting as a
    miss: the host image just written is authoritative, newest token included."""
    capacity = coordinator.padded_buffer_size
    coordinator.req_to_device_buffer[row, :capacity] = slots
    coordinator.req_device_buffer_size[row] = capacity
    coordinator.req_device_buffer_tokens[:, row, :].fill_(-1)
    coordinator.req_device_buffer_token_locs[:, row, :capacity] = slots
    coordinator.lru_slots[:, row, :].copy_(coordinator._lru_init)
    coordinator.spec_swap.reset(row)
    coordinator._skip_first_backup[row] = True


def _device_planes(pool):
    planes = []
    for layer in range(pool.start_layer, pool.end_layer):
        planes += [pool.get_key_buffer(layer), pool.get_value_buffer(layer)]
    return planes


def _restore_history(coordinator, pool, host, destination):
    """Host rows ``host`` -> device slots ``destination`` for every layer's K and V."""
    host_pool = coordinator.mem_pool_host
    all_layers = getattr(host_pool, "load_to_device_all_layer", None)
    if all_layers is not None:
        all_layers(pool, host, destination, io_backend="kernel")
        return
    for layer in range(pool.start_layer, pool.end_layer):
        host_pool.load_to_device_per_layer(pool, host, destination, layer, io_backend="kernel")


def _copy_newest_token(pool, source, target):
    """Rows ``source`` -> ``target`` (one slot each) in every plane: two launches of the
    row-copy kernel through a small device buffer."""
    import torch

    from ._lib import MAX_PLANES
    from .host_pool import pack_rows, unpack_rows

    planes = [p.view(p.shape[0], -1) for p in _device_planes(pool)]
    row_bytes = planes[0][0].numel() * planes[0].element_size()
    staging = torch.empty((len(planes), row_bytes), dtype=torch.uint8, device=planes[0].device)
    src = source.to(planes[0].device, torch.int64).contiguous()
    dst = target.to(planes[0].device, torch.int64).contiguous()
    bytes_planes = [p.view(torch.uint8).view(p.shape[0], row_bytes) for p in planes]
    for first in range(0, len(planes), MAX_PLANES):
        chunk = bytes_planes[first:first + MAX_PLANES]
        stage = staging[first:first + len(chunk)]
        pack_rows(chunk, src, stage, stage_plane_stride=row_bytes)
        unpack_rows(chunk, dst, stage, stage_plane_stride=row_bytes)


# --------------------------------------------------------------------------- demotion

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
    pool = coordinator.mem_pool_device
    page_size = pool.page_size
    if coordinator.padded_buffer_size % page_size:
        raise RuntimeError("Hot buffer must be page-aligned")
    logical = coordinator.req_to_token_pool.req_to_token[row, :length].clone()
    physical = pool.translate_loc_from_full_to_hisparse_device(logical)
    page_ids = _physical_pages(physical, page_size)
    kept, released = plan_demote_pages(getattr(pool, "adaptive_vmm", None), page_ids,
                                       coordinator.padded_buffer_size // page_size)
    position = {page: index for index, page in enumerate(page_ids)}
    prepared = PreparedDemotion(coordinator, req, row, logical, physical, length,
                                tuple(position[page] for page in kept),
                                tuple(position[page] for page in released))
    coordinator.wait_for_pending_backup()
    synchronize()
    shadow = getattr(coordinator.token_to_kv_pool_allocator._kvcache, "_ekv_shadow", None)
    if shadow is not None:
        shadow.check_complete(pool, logical, physical, "demote_source")
    host_pool = coordinator.mem_pool_host
    try:
        host = host_pool.alloc_paged_token_slots(
            coordinator.req_to_host_pool, coordinator.req_to_host_pool_allocated_len, row, 0, length)
        host_pool.backup_from_device_all_layer(pool, host, physical, io_backend="kernel")
        synchronize()
    except Exception:
        # A failed synchronize may leave device work referencing the host rows;
        # the fail-stop path owns them then.
        synchronize()
        _release_host(coordinator, row)
        raise
    return prepared


def abort_demote(prepared):
    """Undo a prepared demotion after the ranks reject it."""
    prepared._check_abortable()
    _release_host(prepared.coordinator, prepared.row)
    prepared.status = _ABORTED


@profile_range("hisparse/demotion/commit")
def commit_demote(prepared, publish_host_backed, synchronize, trim_quiescent=None):
    """Hand the kept pages to the fixed hot buffer and free the rest.

    ``publish_host_backed`` removes the row from resident dispatch; scheduling
    stays paused until every TP rank confirms.
    """
    prepared._enter_commit()
    coordinator = prepared.coordinator
    pool = coordinator.mem_pool_device
    starts = prepared.physical[::pool.page_size]
    hot = _page_slots(starts, prepared.retained_rows, pool.page_size)
    _install_hot_buffer(coordinator, prepared.row, hot.to(coordinator.req_to_device_buffer.dtype))
    forget_source = getattr(coordinator, "_ekv_remove_demoted_source", None)
    if forget_source is not None:
        forget_source(prepared.request)
    pool.full_to_hisparse_device_index_mapping[prepared.logical] = 0
    synchronize()
    import torch

    released = torch.as_tensor(prepared.released_rows, device=starts.device, dtype=torch.long)
    coordinator.token_to_kv_pool_allocator.free_hisparse_indices(starts[released])
    synchronize()
    freed_bytes = trim_quiescent() if trim_quiescent is not None else 0
    publish_host_backed(prepared.row)
    prepared.status = _COMMITTED
    return freed_bytes


# --------------------------------------------------------------------------- promotion

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
    tracker = getattr(pool, "adaptive_vmm", None)
    if tracker is None:
        raise RuntimeError("Promotion requires the tracked MiniMax VMM main pool")
    if int(coordinator.req_device_buffer_size[row]) != coordinator.padded_buffer_size:
        raise RuntimeError("Unexpected source hot-buffer capacity")
    coordinator.wait_for_pending_backup()
    synchronize()
    logical = coordinator.req_to_token_pool.req_to_token[row, :length].clone()
    # Until the first backup after demotion, the host image lacks the newest
    # token: it is still only in the hot buffer's decode slot.
    from_host = length if coordinator._skip_first_backup[row] else length - 1
    host = coordinator.req_to_host_pool[row, :from_host]
    if (int(coordinator.req_to_host_pool_allocated_len[row]) < from_host
            or not bool((host >= 0).all())):
        raise RuntimeError("Promotion source is missing committed host KV")
    newest = None
    if from_host < length:
        newest = coordinator.req_to_device_buffer[row, coordinator.device_buffer_size:][:1]
        if not bool((newest > 0).all()):
            raise RuntimeError("Promotion source is missing the latest device token")
    allocator = coordinator.token_to_kv_pool_allocator
    backed_before = tracker.backing.backed_bytes
    page = pool.page_size
    destination = allocator.hisparse_attn_allocator.alloc(-(-length // page) * page)
    if destination is None:
        raise MemoryError("No physical pages available for promotion")
    try:
        _restore_history(coordinator, pool, host, destination[:from_host])
        if newest is not None:
            _copy_newest_token(pool, newest, destination[from_host:from_host + 1])
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
    prepared._check_abortable()
    coordinator = prepared.coordinator
    coordinator.token_to_kv_pool_allocator.free_hisparse_indices(prepared.destination)
    coordinator.mem_pool_device.adaptive_vmm.trim_quiescent()
    prepared.status = _ABORTED


@profile_range("hisparse/promotion/commit")
def commit_promote(prepared, publish_gpu_resident, synchronize):
    """Release the host-backed source and publish the prepopulated resident mapping."""
    prepared._enter_commit()
    coordinator = prepared.coordinator
    pool = coordinator.mem_pool_device
    # Dropping the source (host rows, hot buffer, old mappings) is the residency
    # hook's job when it is installed, so it stays apart from request completion.
    release_source = getattr(coordinator, "_ekv_cleanup_promotion_source", None)
    if release_source is None:
        coordinator.request_finished(prepared.request)
    else:
        release_source(prepared.request)
    pool.full_to_hisparse_device_index_mapping[prepared.logical] = (
        prepared.destination[:len(prepared.logical)])
    synchronize()
    tracker = pool.adaptive_vmm
    tracker.trim_quiescent()
    publish_gpu_resident(prepared.row)
    register = getattr(coordinator, "_ekv_register_promoted_source", None)
    if register is not None:
        register(prepared.request)
    prepared.status = _COMMITTED
    return max(0, tracker.backing.backed_bytes - prepared.backed_before)
