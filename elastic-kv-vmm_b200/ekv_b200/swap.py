"""Hot-buffer swap-in for host-backed requests (sparse decode with misses).

A host-backed request keeps its full history in host memory and a fixed hot
buffer of ``hot`` slots per layer on the device (docs of the reference's
HiSparse mode; the swap itself is SGLang's block swap kernel, called at
adaptive_sparse/request_residency.py:805-809 and :829-832).  One layer of one
decode step is four launches, none of which waits for the host:

1. ``lookup_slots``   Top-K token ids -> hot slots, compacted miss list (R2);
2. ``swap_select``    victims for the misses (clock order, this step's hits
   pinned), residency map and slot -> token table updated;
3. ``promote_rows``   missed rows copied from host history into their slots;
4. mapped gather      Top-K rows read through the updated map.

``HotLayer`` holds one layer's state and runs the four steps; ``SwapStep`` is
the pre-bound form for a hot loop or a CUDA graph; ``SwapPipeline`` runs a
step's layers with each gather overlapped with the next layer's promotion.
"""

from __future__ import annotations

import torch

from ._lib import MAX_PLANES, call, require_cuda, stream_handle, u64_array
from .pipeline import LayerPipeline
from .resident_lookup import LookupPlan
from .sparse_read import PlaneGather
from .virtual_layout import VirtualKVLayout


def _int32(name, tensor, device):
    require_cuda({name: tensor}, device)
    if tensor.dtype != torch.int32 or tensor.stride(-1) != 1:
        raise TypeError(f"{name} must be an int32 tensor with contiguous rows")


def swap_select(res_map, slot_token, hand, slots, miss_list, miss_count, promo_slot):
    """Assign hot slots to the misses of every row (see module docstring, step 2)."""
    device = require_cuda(dict(res_map=res_map))
    for name, t in dict(res_map=res_map, slot_token=slot_token, hand=hand, slots=slots,
                        miss_list=miss_list, miss_count=miss_count, promo_slot=promo_slot).items():
        _int32(name, t, device)
    batch, k = slots.shape
    if not (res_map.shape[0] == slot_token.shape[0] == hand.numel() == batch == miss_count.numel()):
        raise ValueError("row counts differ")
    call("ekv_swap_select", res_map.data_ptr(), res_map.stride(0), res_map.shape[1],
         slot_token.data_ptr(), slot_token.stride(0), slot_token.shape[1], hand.data_ptr(),
         slots.data_ptr(), slots.stride(0), k, miss_list.data_ptr(), miss_list.stride(0),
         miss_count.data_ptr(), promo_slot.data_ptr(), promo_slot.stride(0), batch,
         device.index, stream_handle(device))


def promote_rows(history_planes, hot_planes, layout, history_rows, miss_list, miss_count, promo_slot):
    """Copy every assigned miss from host history into its hot slot, in every plane.

    ``history_planes[p]`` is [batch * history_rows, row] (pinned host or device
    memory); ``hot_planes[p]`` is a fixed-position region laid out by
    ``layout`` (sink chunk, then one ``layout.request_bytes`` region per row).
    """
    history_planes, hot_planes = list(history_planes), list(hot_planes)
    if not 1 <= len(hot_planes) == len(history_planes) <= MAX_PLANES:
        raise ValueError("need 1..EKV_MAX_PLANES history / hot plane pairs")
    device = require_cuda(dict(miss_list=miss_list))
    for name, t in dict(miss_list=miss_list, miss_count=miss_count, promo_slot=promo_slot).items():
        _int32(name, t, device)
    for h in history_planes:
        if h.device.type == "cpu" and not h.is_pinned():
            raise ValueError("host history must be pinned memory")
    batch, k = miss_list.shape
    call("ekv_promote_rows", u64_array(h.data_ptr() for h in history_planes),
         u64_array(h.data_ptr() for h in hot_planes), len(hot_planes), layout.row_bytes, history_rows,
         layout.chunk_bytes, layout.request_bytes, miss_list.data_ptr(), miss_list.stride(0),
         miss_count.data_ptr(), promo_slot.data_ptr(), promo_slot.stride(0), batch, k,
         device.index, stream_handle(device))


class HotLayer:
    """One layer's hot buffers for ``batch`` host-backed requests.

    ``planes`` are the layer's K and V hot pools, each a flat tensor laid out by
    ``VirtualKVLayout(batch, hot, row_elements)`` (sink chunk, then one region
    of ``hot`` rows per request).  ``res_map[b, t]`` is token t's hot slot or
    -1; ``slot_token[b, s]`` is the token in slot s or -1; ``hand[b]`` is the
    clock position victim search starts from.
    """

    def __init__(self, batch, context, hot, row_elements, device, dtype=torch.bfloat16, planes=None,
                 chunk_bytes=2 << 20):
        self.device = torch.device(device)
        self.layout = VirtualKVLayout(batch, hot, row_elements, itemsize=torch.empty((), dtype=dtype).element_size(),
                                      chunk_bytes=chunk_bytes)
        elems = self.layout.capacity_bytes // self.layout.itemsize
        self.planes = planes if planes is not None else [torch.zeros(elems, dtype=dtype, device=self.device)
                                                         for _ in range(2)]
        self.batch, self.context, self.hot = batch, context, hot
        self.res_map = torch.full((batch, context), -1, dtype=torch.int32, device=self.device)
        self.slot_token = torch.full((batch, hot), -1, dtype=torch.int32, device=self.device)
        self.hand = torch.zeros(batch, dtype=torch.int32, device=self.device)

    def step(self, topk, history_planes, outputs, *, request_ids=None):
        """Lookup, swap-in and gather for Top-K ``topk`` [batch, k] (int32 token ids)."""
        plan = SwapStep(self, topk, history_planes, outputs, request_ids=request_ids)
        plan()
        return plan


class SwapStep:
    """The four launches of one layer's decode step, pre-bound to fixed tensors.

    After a call: ``lookup`` holds this step's hit slots / miss list (before the
    swap), ``promo_slot`` the slot given to each miss, ``outputs`` the gathered
    K and V rows (every valid Top-K token is resident after the swap).
    """

    def __init__(self, layer: HotLayer, topk, history_planes, outputs, *, request_ids=None):
        dev = layer.device
        batch, k = topk.shape
        _int32("topk", topk, dev)
        self.layer = layer
        self.lookup = LookupPlan(layer.res_map, topk)
        self.promo_slot = torch.empty((batch, k), dtype=torch.int32, device=dev)
        self.history_planes = list(history_planes)
        for h in self.history_planes:
            if h.device.type == "cpu" and not h.is_pinned():
                raise ValueError("host history must be pinned memory")
        self.request_ids = request_ids if request_ids is not None else torch.arange(batch, device=dev)
        self.lengths = torch.full((batch,), layer.context, dtype=torch.int64, device=dev)
        width = layer.layout.row_elements
        self.gather = PlaneGather(layer.planes, topk, self.request_ids, self.lengths, layer.res_map, None,
                                  [o.view(batch, k, width) for o in outputs], layer.layout,
                                  indirect=False, mapped=True)
        self._keep = (topk, outputs)
        self._select_args = (
            layer.res_map.data_ptr(), layer.res_map.stride(0), layer.context,
            layer.slot_token.data_ptr(), layer.slot_token.stride(0), layer.hot, layer.hand.data_ptr(),
            self.lookup.slots.data_ptr(), self.lookup.slots.stride(0), k,
            self.lookup.miss_list.data_ptr(), self.lookup.miss_list.stride(0), self.lookup.miss_count.data_ptr(),
            self.promo_slot.data_ptr(), self.promo_slot.stride(0), batch, dev.index,
        )
        self._promote_args = (
            u64_array(h.data_ptr() for h in self.history_planes), u64_array(p.data_ptr() for p in layer.planes),
            len(layer.planes), layer.layout.row_bytes, layer.context, layer.layout.chunk_bytes,
            layer.layout.request_bytes, self.lookup.miss_list.data_ptr(), self.lookup.miss_list.stride(0),
            self.lookup.miss_count.data_ptr(), self.promo_slot.data_ptr(), self.promo_slot.stride(0),
            batch, k, dev.index,
        )
        self.device = dev

    def swap_in(self, stream: int | None = None) -> None:
        """Steps 1-3: lookup, victim selection, promotion (host-link bound)."""
        stream = stream_handle(self.device) if stream is None else stream
        self.lookup(stream)
        call("ekv_swap_select", *self._select_args, stream)
        call("ekv_promote_rows", *self._promote_args, stream)

    def __call__(self, stream: int | None = None) -> None:
        stream = stream_handle(self.device) if stream is None else stream
        self.swap_in(stream)
        self.gather(stream)


class SwapPipeline(LayerPipeline):
    """All layers of a decode step with each layer's gather overlapped with the next
    layer's swap-in.

    ``SwapStep`` runs its four launches in order, so the host-link-bound promotion
    and the HBM-bound gather of a layer never overlap.  Here the lookups, victim
    selections and promotions of all layers run in order on the caller's stream
    and layer i's gather runs on a second stream as soon as layer i's promotion
    is done (one event per layer), while layer i+1 promotes.  The promotion
    kernel's small fixed grid leaves the SMs' other slots to the gather.  The
    gathers stay in layer order on their stream, so layers may share one output
    buffer; the caller's stream waits for the last gather before returning.
    Works eagerly and under CUDA graph capture (the second stream forks from and
    joins the caller's stream).
    """

    def __init__(self, plans):
        self.plans = list(plans)
        if not self.plans:
            raise ValueError("need at least one layer")
        super().__init__([p.swap_in for p in self.plans], [p.gather for p in self.plans], self.plans[0].device)
