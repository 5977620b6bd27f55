// Compiled Python binding of the per-call residency lookups and gathers (optional).
//
// resolve_resident, lookup_slots, the batched shared-prefix resolver and
// gather_rows / gather_rows_planes are called once per layer per decode step
// through the reference's Python API.  Through ctypes a call costs ~10 us of
// host time (reading ~30 tensor attributes in Python and marshalling ~28
// arguments); here the tensors arrive as at::Tensor and their pointers,
// strides and the current stream are read in C++.  The kernels are reached
// through the SAME C entry points of libekv_b200.so: Python hands over their
// addresses once (bind), so this module does not link against the library.
//
// Only the well-formed calls are handled here: every tensor on one CUDA
// device, supported dtypes and shapes.  Anything else returns kNotHandled and
// the Python wrapper runs its checked ctypes path, which raises the documented
// errors -- so error types and messages stay exactly those of the Python API.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include <algorithm>
#include <cstdint>
#include <limits>
#include <optional>
#include <vector>

#include "ekv_kernels.h"

namespace {

constexpr int kNotHandled = 1;  // ask the caller to take its checked path
constexpr int kKernelError = -1;

decltype(&ekv_resolve_resident) g_resolve = nullptr;
decltype(&ekv_lookup_slots) g_lookup = nullptr;
decltype(&ekv_resolve_shared_blocks) g_shared = nullptr;
decltype(&ekv_gather_rows) g_gather = nullptr;
decltype(&ekv_gather_rows_planes) g_gather_planes = nullptr;

void bind(int64_t resolve, int64_t lookup, int64_t shared, int64_t gather, int64_t gather_planes) {
    g_resolve = reinterpret_cast<decltype(&ekv_resolve_resident)>(resolve);
    g_lookup = reinterpret_cast<decltype(&ekv_lookup_slots)>(lookup);
    g_shared = reinterpret_cast<decltype(&ekv_resolve_shared_blocks)>(shared);
    g_gather = reinterpret_cast<decltype(&ekv_gather_rows)>(gather);
    g_gather_planes = reinterpret_cast<decltype(&ekv_gather_rows_planes)>(gather_planes);
}

int index_size(const at::Tensor& t) {
    switch (t.scalar_type()) {
        case at::kInt: return 4;
        case at::kLong: return 8;
        default: return 0;
    }
}

// All defined tensors CUDA on one device; the device index, or -1.
int common_device(std::initializer_list<const at::Tensor*> tensors) {
    int device = -1;
    for (const at::Tensor* t : tensors) {
        if (!t || !t->defined()) continue;
        if (!t->is_cuda()) return -1;
        const int here = t->get_device();
        if (device < 0) {
            device = here;
        } else if (here != device) {
            return -1;
        }
    }
    return device;
}

void* stream_of(int device) { return c10::cuda::getCurrentCUDAStream(device).stream(); }

int resolve_resident(const at::Tensor& topk, const at::Tensor& table, const at::Tensor& mapping,
                     const at::Tensor& rows, const at::Tensor& lengths, const at::Tensor& selected,
                     const at::Tensor& output, int64_t block_size) {
    if (!g_resolve || topk.dim() != 3) return kNotHandled;
    const int64_t width = topk.size(2) * block_size;
    if (selected.numel() == 0 || width == 0) return 0;  // no-op, as the reference
    const int device = common_device({&topk, &table, &mapping, &rows, &lengths, &selected, &output});
    if (device < 0 || output.scalar_type() != at::kInt || table.dim() != 2 || output.dim() != 3) return kNotHandled;
    const int es_topk = index_size(topk), es_table = index_size(table), es_map = index_size(mapping);
    const int es_rows = index_size(rows), es_len = index_size(lengths), es_sel = index_size(selected);
    if (!es_topk || !es_table || !es_map || !es_rows || !es_len || !es_sel) return kNotHandled;
    const int rc = g_resolve(
        topk.data_ptr(), es_topk, topk.stride(1), topk.stride(2), topk.size(2),
        table.data_ptr(), es_table, table.stride(0), table.stride(1),
        mapping.data_ptr(), es_map, mapping.stride(0),
        rows.data_ptr(), es_rows, rows.stride(0),
        lengths.data_ptr(), es_len, lengths.stride(0),
        selected.data_ptr(), es_sel, selected.stride(0), selected.numel(),
        output.data_ptr<int32_t>(), output.stride(1), output.stride(2),
        block_size, device, stream_of(device));
    return rc == 0 ? 0 : kKernelError;
}

bool rows_of(const std::optional<at::Tensor>& t, int device, at::ScalarType dtype, int64_t batch) {
    if (!t) return true;
    return t->is_cuda() && t->get_device() == device && t->scalar_type() == dtype && t->dim() >= 1 &&
           t->size(0) == batch && t->stride(-1) == 1;
}

// Returns (status, slots, miss, miss_list, miss_count); outputs not given are allocated.
py::tuple lookup_slots(const at::Tensor& residency_map, const at::Tensor& topk,
                       const std::optional<at::Tensor>& lengths, std::optional<at::Tensor> slots,
                       std::optional<at::Tensor> miss, std::optional<at::Tensor> miss_list,
                       std::optional<at::Tensor> miss_count, bool compact) {
    auto not_handled = [] { return py::make_tuple(kNotHandled, py::none(), py::none(), py::none(), py::none()); };
    if (!g_lookup || residency_map.dim() != 2 || topk.dim() != 2 || residency_map.size(0) != topk.size(0)) {
        return not_handled();
    }
    const at::Tensor* len_ptr = lengths ? &*lengths : nullptr;
    const int device = common_device({&residency_map, &topk, len_ptr});
    if (device < 0 || residency_map.stride(1) != 1 || topk.stride(1) != 1) return not_handled();
    const int es_map = index_size(residency_map), es_topk = index_size(topk);
    const int es_len = lengths ? index_size(*lengths) : 4;
    if (!es_map || !es_topk || !es_len) return not_handled();
    const int64_t batch = topk.size(0), k = topk.size(1);
    if (lengths && (lengths->dim() != 1 || lengths->size(0) != batch || lengths->stride(0) != 1)) {
        return not_handled();
    }
    const auto options = residency_map.options();
    if (!slots) slots = at::empty({batch, k}, options.dtype(at::kInt));
    if (!miss) miss = at::empty({batch, k}, options.dtype(at::kBool));
    if (compact) {
        if (!miss_list) miss_list = at::empty({batch, k}, options.dtype(at::kInt));
        if (!miss_count) miss_count = at::empty({batch}, options.dtype(at::kInt));
    }
    if (!rows_of(slots, device, at::kInt, batch) || !rows_of(miss, device, at::kBool, batch) ||
        !rows_of(miss_list, device, at::kInt, batch) || !rows_of(miss_count, device, at::kInt, batch) ||
        (miss_count && miss_count->numel() != batch)) {
        return not_handled();
    }
    const int rc = g_lookup(
        residency_map.data_ptr(), es_map, residency_map.stride(0), residency_map.size(1),
        topk.data_ptr(), es_topk, topk.stride(0),
        lengths ? lengths->data_ptr() : nullptr, es_len,
        batch, k,
        slots->data_ptr<int32_t>(), slots->stride(0),
        reinterpret_cast<uint8_t*>(miss->data_ptr()), miss->stride(0),
        miss_list ? miss_list->data_ptr<int32_t>() : nullptr, miss_list ? miss_list->stride(0) : 0,
        miss_count ? miss_count->data_ptr<int32_t>() : nullptr,
        device, stream_of(device));
    auto opt = [](const std::optional<at::Tensor>& t) { return t ? py::cast(*t) : py::none(); };
    return py::make_tuple(rc == 0 ? 0 : kKernelError, py::cast(*slots), py::cast(*miss), opt(miss_list),
                          opt(miss_count));
}

// Exact Python ints only (bool and int subclasses take the checked path); false
// when an element is not one, overflows int64 or falls outside [lo, hi).
bool int_list(const py::sequence& seq, int64_t lo, int64_t hi, std::vector<int64_t>& out) {
    const size_t n = py::len(seq);
    out.resize(n);
    for (size_t i = 0; i < n; ++i) {
        PyObject* item = PySequence_GetItem(seq.ptr(), static_cast<Py_ssize_t>(i));
        if (!item) {
            PyErr_Clear();
            return false;
        }
        const bool exact = PyLong_CheckExact(item);
        int overflow = 0;
        const long long value = exact ? PyLong_AsLongLongAndOverflow(item, &overflow) : 0;
        Py_DECREF(item);
        if (!exact || overflow || value < lo || value >= hi) {
            PyErr_Clear();
            return false;
        }
        out[i] = value;
    }
    return true;
}

// resolve_shared_block_locations_batched: (status, valid, physical).
py::tuple shared_blocks(const at::Tensor& block_ids, const py::sequence& source_rows, const at::Tensor& seq_len,
                        const py::sequence& shared_tokens, int64_t block_size, const at::Tensor& table,
                        const at::Tensor& mapping, bool exclude_newest, std::optional<at::Tensor> masked) {
    auto not_handled = [] { return py::make_tuple(kNotHandled, py::none(), py::none()); };
    if (!g_shared || block_ids.dim() != 2 || block_size < 1 || block_size > (int64_t{1} << 30) ||
        table.dim() != 2 || table.size(1) == 0 || mapping.dim() != 1 || mapping.numel() == 0 ||
        seq_len.dim() != 1) {
        return not_handled();
    }
    const int64_t requests = block_ids.size(0), per_request = block_ids.size(1);
    const at::Tensor* masked_ptr = masked ? &*masked : nullptr;
    const int device = common_device({&block_ids, &seq_len, &table, &mapping, masked_ptr});
    const int es_blocks = index_size(block_ids), es_len = index_size(seq_len);
    const int es_table = index_size(table), es_map = index_size(mapping);
    if (device < 0 || requests == 0 || per_request == 0 || requests > EKV_SHARED_INLINE_MAX || !es_blocks ||
        !es_len || !es_table || !es_map || seq_len.numel() != requests) {
        return not_handled();
    }
    if (masked && (masked->sizes() != block_ids.sizes() || masked->scalar_type() != block_ids.scalar_type() ||
                   masked->strides() != block_ids.strides())) {
        return not_handled();
    }
    std::vector<int64_t> rows, prefixes;
    if (!int_list(source_rows, 0, table.size(0), rows) ||
        !int_list(shared_tokens, 0, std::numeric_limits<int64_t>::max(), prefixes) ||
        static_cast<int64_t>(rows.size()) != requests || static_cast<int64_t>(prefixes.size()) != requests) {
        return not_handled();
    }
    const auto options = block_ids.options();
    at::Tensor valid = at::empty({requests, per_request}, options.dtype(at::kBool));
    at::Tensor physical = at::empty({requests, per_request, block_size}, options.dtype(at::kInt));
    const int rc = g_shared(
        block_ids.data_ptr(), es_blocks, requests, per_request, block_ids.stride(0), block_ids.stride(1),
        rows.data(), 0, prefixes.data(), 0, seq_len.data_ptr(), es_len, seq_len.stride(0), block_size,
        table.data_ptr(), es_table, table.size(0), table.size(1), table.stride(0), table.stride(1),
        mapping.data_ptr(), es_map, mapping.numel(), mapping.stride(0), 1,
        reinterpret_cast<uint8_t*>(valid.data_ptr()), physical.data_ptr<int32_t>(),
        masked ? masked->data_ptr() : nullptr, exclude_newest ? 1 : 0, device, stream_of(device));
    return py::make_tuple(rc == 0 ? 0 : kKernelError, valid, physical);
}

// Index tensors of a gather: positions [B, S], request_ids / lengths [B], and the
// table / slot offsets the addressing mode uses (mode 0 direct, 1 indirect, 2
// mapped).  Every given tensor CUDA on one device and contiguous (the Python
// API checks the unused table too); element sizes of the used ones in `es`.
struct GatherIndex {
    int device = -1;
    int es[5] = {0, 0, 0, 8, 8};  // positions, request_ids, lengths, table, offsets
    const void* table = nullptr;
    const void* offsets = nullptr;
};

bool gather_index(const at::Tensor& positions, const at::Tensor& request_ids, const at::Tensor& lengths,
                  const std::optional<at::Tensor>& request_table, const std::optional<at::Tensor>& slot_offsets,
                  int mode, GatherIndex& out) {
    const at::Tensor* table = request_table ? &*request_table : nullptr;
    const at::Tensor* offsets = slot_offsets ? &*slot_offsets : nullptr;
    out.device = common_device({&positions, &request_ids, &lengths, table, offsets});
    if (out.device < 0) return false;
    for (const at::Tensor* t : {&positions, &request_ids, &lengths, table, offsets}) {
        if (t && !t->is_contiguous()) return false;
    }
    if ((mode >= 1 && !table) || (mode == 1 && !offsets)) return false;
    out.es[0] = index_size(positions);
    out.es[1] = index_size(request_ids);
    out.es[2] = index_size(lengths);
    if (mode >= 1) {
        out.es[3] = index_size(*table);
        out.table = table->data_ptr();
    }
    if (mode == 1) {
        out.es[4] = index_size(*offsets);
        out.offsets = offsets->data_ptr();
    }
    for (int e : out.es) {
        if (!e) return false;
    }
    return true;
}

bool rows_shape(const at::Tensor& t, int64_t batch, int64_t selected, int64_t width) {
    return t.dim() == 3 && t.size(0) == batch && t.size(1) == selected && t.size(2) == width;
}

// gather_rows (the reference's single-plane call).
int gather_rows(const at::Tensor& raw, const at::Tensor& positions, const at::Tensor& request_ids,
                const at::Tensor& lengths, const std::optional<at::Tensor>& request_table,
                const std::optional<at::Tensor>& slot_offsets, const at::Tensor& output, int64_t width,
                int64_t table_width, int64_t request_stride, int64_t sink_elements, bool indirect) {
    if (!g_gather || positions.dim() != 2) return kNotHandled;
    const int64_t batch = positions.size(0), selected = positions.size(1);
    if (!rows_shape(output, batch, selected, width)) return kNotHandled;
    if (batch == 0 || selected == 0) return 0;  // no-op, as the reference
    const int mode = indirect ? 1 : 0;
    GatherIndex ix;
    if (!gather_index(positions, request_ids, lengths, request_table, slot_offsets, mode, ix)) return kNotHandled;
    if (common_device({&raw, &output}) != ix.device || !raw.is_contiguous() || !output.is_contiguous() ||
        raw.scalar_type() != output.scalar_type()) {
        return kNotHandled;
    }
    const int rc = g_gather(
        raw.data_ptr(), output.data_ptr(), raw.element_size(), positions.data_ptr(), ix.es[0],
        request_ids.data_ptr(), ix.es[1], lengths.data_ptr(), ix.es[2], ix.table, ix.es[3], ix.offsets, ix.es[4],
        batch, selected, width, table_width, request_stride, sink_elements, mode, ix.device, stream_of(ix.device));
    return rc == 0 ? 0 : kKernelError;
}

// gather_rows_planes: one row selection over every plane, EKV_MAX_PLANES planes per launch.
int gather_rows_planes(const std::vector<at::Tensor>& planes, const std::vector<at::Tensor>& outputs,
                       const at::Tensor& positions, const at::Tensor& request_ids, const at::Tensor& lengths,
                       const std::optional<at::Tensor>& request_table,
                       const std::optional<at::Tensor>& slot_offsets, int64_t width, int64_t max_tokens,
                       int64_t request_stride, int64_t sink_elements, bool indirect, bool mapped) {
    if (!g_gather_planes || planes.size() != outputs.size() || positions.dim() != 2 || (indirect && mapped)) {
        return kNotHandled;
    }
    const int64_t batch = positions.size(0), selected = positions.size(1);
    for (const at::Tensor& out : outputs) {
        if (!rows_shape(out, batch, selected, width)) return kNotHandled;
    }
    if (planes.empty() || batch == 0 || selected == 0) return 0;
    const int mode = mapped ? 2 : (indirect ? 1 : 0);
    GatherIndex ix;
    if (!gather_index(positions, request_ids, lengths, request_table, slot_offsets, mode, ix)) return kNotHandled;
    const at::ScalarType dtype = planes[0].scalar_type();
    for (size_t p = 0; p < planes.size(); ++p) {
        const at::Tensor& src = planes[p];
        const at::Tensor& dst = outputs[p];
        if (common_device({&src, &dst}) != ix.device || !src.is_contiguous() || !dst.is_contiguous() ||
            src.scalar_type() != dtype || dst.scalar_type() != dtype) {
            return kNotHandled;
        }
    }
    // A residency map is indexed by token: its row width is the map's, not the layout's.
    const int64_t table_width = mode == 2 ? request_table->size(-1) : max_tokens;
    const int64_t itemsize = planes[0].element_size();
    void* stream = stream_of(ix.device);
    uint64_t src[EKV_MAX_PLANES], dst[EKV_MAX_PLANES];
    for (size_t start = 0; start < planes.size(); start += EKV_MAX_PLANES) {
        const int n = static_cast<int>(std::min<size_t>(EKV_MAX_PLANES, planes.size() - start));
        for (int p = 0; p < n; ++p) {
            src[p] = reinterpret_cast<uint64_t>(planes[start + p].data_ptr());
            dst[p] = reinterpret_cast<uint64_t>(outputs[start + p].data_ptr());
        }
        const int rc = g_gather_planes(
            src, dst, n, itemsize, positions.data_ptr(), ix.es[0], request_ids.data_ptr(), ix.es[1],
            lengths.data_ptr(), ix.es[2], ix.table, ix.es[3], ix.offsets, ix.es[4], batch, selected, width,
            table_width, request_stride, sink_elements, mode, ix.device, stream);
        if (rc != 0) return kKernelError;
    }
    return 0;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "Compiled binding of the per-call residency lookups of libekv_b200.so";
    m.def("bind", &bind, "set the addresses of the C entry points");
    m.def("resolve_resident", &resolve_resident);
    m.def("lookup_slots", &lookup_slots, py::arg("residency_map"), py::arg("topk"), py::arg("lengths"),
          py::arg("slots"), py::arg("miss"), py::arg("miss_list"), py::arg("miss_count"), py::arg("compact"));
    m.def("shared_blocks", &shared_blocks);
    m.def("gather_rows", &gather_rows);
    m.def("gather_rows_planes", &gather_rows_planes);
    m.attr("NOT_HANDLED") = kNotHandled;
    m.attr("KERNEL_ERROR") = kKernelError;
}
