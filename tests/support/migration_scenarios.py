"""Migration transaction scenarios and the state trace they record.

``run_all(make_world, migration)`` drives a migration module -- the reference's
adaptive_sparse/migration.py (in tests/golden/make_golden.py, on the CPU world
of ``standin``) or this package's ``ekv_b200.migration`` (in the GPU test) --
through the same sequence of demotions, promotions, aborts and rejected calls,
and records after every step the state the transactions are responsible for:

* the prepared records (retained / released page rows, status);
* the coordinator's per-request tables (host rows, hot buffer, its token
  locations and LRU slots, the first-backup flag);
* the published logical -> physical mapping of the request's tokens;
* the page tracker (owned pages, per-chunk references) and the backing's
  mapped chunks;
* the allocator's free list and every page set it was asked to free;
* return values (released / grown bytes) and published rows;
* whether every moved row holds the bytes it should (host rows after
  demotion, destination rows after promotion).

The trace is JSON; parity is trace equality.
"""

from __future__ import annotations

import os
from types import SimpleNamespace

import torch

from .standin import install_request, payload

GEOMETRY = dict(layers=2, heads=8, head_dim=128, page_size=16, pages=512, rows=4, hot_capacity=64,
                host_rows=8192, table_width=8192)
ROW, LENGTH, SEED = 1, 2000, 3


def _ints(t):
    return [int(v) for v in t.reshape(-1).tolist()]


def _record(world, row, logical, **extra):
    c, tracker = world.coordinator, world.tracker
    cap = c.padded_buffer_size
    n_host = int(c.req_to_host_pool_allocated_len[row])
    state = dict(
        host_rows=_ints(c.req_to_host_pool[row, :max(n_host, 1)]),
        host_allocated=n_host,
        hot_buffer=_ints(c.req_to_device_buffer[row, :cap]),
        hot_size=int(c.req_device_buffer_size[row]),
        hot_tokens_cleared=bool((c.req_device_buffer_tokens[:, row, :] == -1).all()),
        hot_token_locs=_ints(c.req_device_buffer_token_locs[:, row, :cap]),
        lru=_ints(c.lru_slots[:, row, :]),
        skip_first_backup=bool(c._skip_first_backup[row]),
        mapping=_ints(world.pool.full_to_hisparse_device_index_mapping[logical]),
        owned_pages=sorted(int(p) for p in tracker.pages),
        refs=sorted([int(k), int(v)] for k, v in tracker.refs.items()),
        mapped_chunks=sorted(int(x) for x in world.backing.mapped_chunks),
        free_pages=list(world.physical.free_pages),
        freed=[list(x) for x in c.token_to_kv_pool_allocator.freed],
        host_free=int(world.host.available_size()),
    )
    state.update(extra)
    return state


def _rows_hold(world, plane_slots, want_slots, seed):
    """Every plane's rows at ``plane_slots`` hold the payload written for ``want_slots``."""
    ok = True
    for p, view in enumerate(world.views):
        got = view.view(view.shape[0], -1).view(torch.int16)[plane_slots.to(view.device).long()]
        ok &= bool(torch.equal(got, payload(p + 100 * seed, want_slots.to(view.device), world.width)))
    return ok


def _host_holds(world, host_rows, source_slots, seed):
    ok = True
    for p in range(len(world.views)):
        got = world.host.plane_view(p)[host_rows.cpu().long()].cpu().view(torch.int16)
        ok &= bool(torch.equal(got, payload(p + 100 * seed, source_slots.cpu(), world.width)))
    return ok


def _setup(make_world):
    """World with two other requests' pages around the migrated request's, so chunks
    are shared and chunk-aware retention has choices to make."""
    world = make_world(**GEOMETRY)
    c = world.coordinator
    other_a = world.physical.alloc(30 * world.page)
    world.physical.alloc(40 * world.page)  # request B keeps its pages
    c.token_to_kv_pool_allocator.free_hisparse_indices(other_a[: 12 * world.page])  # A frees pages 1..12
    c.token_to_kv_pool_allocator.freed.clear()
    # The migrated request's 125 pages, in token order: 34 in chunk 2 of every plane
    # (pages 128..191, no other owner), then 12 and 57 pages in chunks 0 and 1 (shared
    # with the sink and request B), then 22 more in chunk 2.
    order = [*range(150, 184), *range(1, 13), *range(71, 128), *range(128, 150)]
    world.physical.free_pages = order + [p for p in world.physical.free_pages if p not in set(order)]
    req, slots, logical = install_request(world, ROW, LENGTH, seed=SEED)
    return world, req, slots, logical


def _prepared(record):
    if hasattr(record, "retained_rows"):
        return dict(retained_rows=list(record.retained_rows), released_rows=list(record.released_rows),
                    committed_len=record.committed_len, status=record.status)
    return dict(destination=_ints(record.destination), status=record.status)


def round_trip(make_world, migration, aware, newest_on_device=False):
    """prepare_demote -> commit_demote -> (one decode step) -> prepare_promote -> commit_promote."""
    os.environ["EKV_CHUNK_AWARE_RETENTION"] = "1" if aware else "0"
    world, req, slots, logical = _setup(make_world)
    c, sync, trace, published = world.coordinator, world.sync, [], []
    try:
        demotion = migration.prepare_demote(c, req, sync)
        host = c.req_to_host_pool[ROW, :LENGTH]
        trace.append(_record(world, ROW, logical, step="prepare_demote", prepared=_prepared(demotion),
                             host_holds_source=_host_holds(world, host, slots, SEED)))
        freed_bytes = migration.commit_demote(demotion, published.append, sync,
                                              trim_quiescent=world.tracker.trim_quiescent)
        trace.append(_record(world, ROW, logical, step="commit_demote", prepared=_prepared(demotion),
                             returned=int(freed_bytes), published=list(published)))
        length = LENGTH
        sources = slots
        if newest_on_device:
            # One decode step after the demotion: the newest token lives only in the hot
            # buffer's decode slot until the next backup.
            newest_slot = c.req_to_device_buffer[ROW, c.device_buffer_size:c.device_buffer_size + 1].clone()
            c._skip_first_backup[ROW] = False
            newest_logical = logical[-1:] + 7
            c.req_to_token_pool.req_to_token[ROW, length] = newest_logical[0]
            length += 1
            req.kv.kv_committed_len = req.kv.kv_allocated_len = length
            logical = torch.cat([logical, newest_logical])
            sources = torch.cat([slots, newest_slot.to(slots.device)])
        promotion = migration.prepare_promote(c, req, sync)
        destination = promotion.destination[:length]
        trace.append(_record(world, ROW, logical, step="prepare_promote", prepared=_prepared(promotion),
                             destination_holds_source=_rows_hold(world, destination, sources, SEED)))
        grown = migration.commit_promote(promotion, published.append, sync)
        trace.append(_record(world, ROW, logical, step="commit_promote", prepared=_prepared(promotion),
                             returned=int(grown), published=list(published)))
    finally:
        os.environ.pop("EKV_CHUNK_AWARE_RETENTION", None)
        world.close()
    return trace


def aborts(make_world, migration):
    """abort_demote, then a committed demotion whose promotion is aborted and redone."""
    os.environ["EKV_CHUNK_AWARE_RETENTION"] = "1"
    world, req, slots, logical = _setup(make_world)
    c, sync, trace, published = world.coordinator, world.sync, [], []
    try:
        first = migration.prepare_demote(c, req, sync)
        migration.abort_demote(first)
        trace.append(_record(world, ROW, logical, step="abort_demote", prepared=_prepared(first)))
        demotion = migration.prepare_demote(c, req, sync)
        migration.commit_demote(demotion, published.append, sync, trim_quiescent=world.tracker.trim_quiescent)
        promotion = migration.prepare_promote(c, req, sync)
        migration.abort_promote(promotion)
        trace.append(_record(world, ROW, logical, step="abort_promote", prepared=_prepared(promotion)))
        again = migration.prepare_promote(c, req, sync)
        trace.append(_record(world, ROW, logical, step="prepare_promote_again", prepared=_prepared(again),
                             destination_holds_source=_rows_hold(world, again.destination[:LENGTH], slots, SEED)))
        grown = migration.commit_promote(again, published.append, sync)
        trace.append(_record(world, ROW, logical, step="commit_promote", returned=int(grown),
                             published=list(published)))
    finally:
        os.environ.pop("EKV_CHUNK_AWARE_RETENTION", None)
        world.close()
    return trace


def _outcome(fn):
    try:
        fn()
    except Exception as exc:  # the type and message are the contract
        return [type(exc).__name__, str(exc)]
    return ["ok", ""]


def rejections(make_world, migration):
    """Calls the transactions must refuse, with the exception type and message of each."""
    out = {}
    world, req, slots, logical = _setup(make_world)
    c, sync, pool = world.coordinator, world.sync, world.pool
    mapping = pool.full_to_hisparse_device_index_mapping
    try:
        c.spec_swap.enabled = True
        out["demote_with_speculation"] = _outcome(lambda: migration.prepare_demote(c, req, sync))
        c.spec_swap.enabled = False
        short = SimpleNamespace(kv=SimpleNamespace(req_pool_idx=ROW, kv_committed_len=c.padded_buffer_size - 1,
                                                   kv_allocated_len=c.padded_buffer_size - 1),
                                hisparse_staging=False)
        out["demote_short_request"] = _outcome(lambda: migration.prepare_demote(c, short, sync))
        staging = SimpleNamespace(kv=req.kv, hisparse_staging=True)
        out["demote_staging_request"] = _outcome(lambda: migration.prepare_demote(c, staging, sync))
        c.req_device_buffer_size[ROW] = 5
        out["demote_with_hot_state"] = _outcome(lambda: migration.prepare_demote(c, req, sync))
        c.req_device_buffer_size[ROW] = 0
        saved = mapping[logical].clone()
        mapping[logical[100]] = 0
        out["demote_missing_location"] = _outcome(lambda: migration.prepare_demote(c, req, sync))
        mapping[logical] = saved
        mapping[logical[world.page * 3]] = saved[world.page * 3] + 1  # page start off the page grid
        out["demote_misaligned_page"] = _outcome(lambda: migration.prepare_demote(c, req, sync))
        mapping[logical] = saved
        mapping[logical[world.page * 5:world.page * 6]] = saved[world.page * 2:world.page * 3]
        out["demote_reused_page"] = _outcome(lambda: migration.prepare_demote(c, req, sync))
        mapping[logical] = saved
        out["state_after_rejected_demotions"] = _record(world, ROW, logical)
        demotion = migration.prepare_demote(c, req, sync)
        migration.commit_demote(demotion, lambda row: None, sync, trim_quiescent=world.tracker.trim_quiescent)
        out["commit_demote_twice"] = _outcome(
            lambda: migration.commit_demote(demotion, lambda row: None, sync))
        out["abort_committed_demotion"] = _outcome(lambda: migration.abort_demote(demotion))
        c.compress_ratio = 2
        out["promote_compressed"] = _outcome(lambda: migration.prepare_promote(c, req, sync))
        c.compress_ratio = 1
        c.req_device_buffer_size[ROW] = 7
        out["promote_wrong_hot_capacity"] = _outcome(lambda: migration.prepare_promote(c, req, sync))
        c.req_device_buffer_size[ROW] = c.padded_buffer_size
        kept = c.req_to_host_pool[ROW, 10].clone()
        c.req_to_host_pool[ROW, 10] = -1
        out["promote_missing_host_row"] = _outcome(lambda: migration.prepare_promote(c, req, sync))
        c.req_to_host_pool[ROW, 10] = kept
        c._skip_first_backup[ROW] = False
        hot = c.req_to_device_buffer[ROW, c.device_buffer_size].clone()
        c.req_to_device_buffer[ROW, c.device_buffer_size] = 0
        out["promote_missing_newest_token"] = _outcome(lambda: migration.prepare_promote(c, req, sync))
        c.req_to_device_buffer[ROW, c.device_buffer_size] = hot
        c._skip_first_backup[ROW] = True
        free_pages = world.physical.free_pages
        world.physical.free_pages = free_pages[:3]
        out["promote_out_of_pages"] = _outcome(lambda: migration.prepare_promote(c, req, sync))
        world.physical.free_pages = free_pages
        out["state_after_rejected_promotions"] = _record(world, ROW, logical)
        promotion = migration.prepare_promote(c, req, sync)
        migration.commit_promote(promotion, lambda row: None, sync)
        out["commit_promote_twice"] = _outcome(lambda: migration.commit_promote(promotion, lambda row: None, sync))
        out["abort_committed_promotion"] = _outcome(lambda: migration.abort_promote(promotion))
    finally:
        world.close()
    return out


def run_all(make_world, migration):
    """Every scenario's trace; ``make_world(**GEOMETRY)`` returns a ``standin`` world with
    a ``sync`` attribute (the synchronize callable the transactions get)."""
    return {
        "plain": round_trip(make_world, migration, aware=False),
        "chunk_aware": round_trip(make_world, migration, aware=True),
        "newest_on_device": round_trip(make_world, migration, aware=True, newest_on_device=True),
        "aborts": aborts(make_world, migration),
        "rejections": rejections(make_world, migration),
    }
