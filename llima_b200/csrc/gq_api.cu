// C ABI of libgguf_b200.so: argument validation, batching by GGML type, and the
// host-buffer session that pipelines host->device copies, kernels and device->host copies.
#include <cuda_runtime.h>

#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <deque>
#include <map>
#include <unordered_map>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include "gq_internal.h"

namespace {

thread_local int g_last_cuda = 0;

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return GQ_OK;
    g_last_cuda = static_cast<int>(e);
    return GQ_ERR_CUDA;
}
int cuda_status(int e) { return cuda_status(static_cast<cudaError_t>(e)); }

// Makes `device` current for one entry-point call and puts the caller's current device
// back on every return path (hosts such as torch keep their own notion of it).
class DeviceScope {
public:
    explicit DeviceScope(int device) {
        status_ = cuda_status(cudaGetDevice(&prev_));
        if (status_ == GQ_OK && prev_ != device) {
            status_ = cuda_status(cudaSetDevice(device));
            switched_ = status_ == GQ_OK;
        }
    }
    ~DeviceScope() {
        if (switched_) cudaSetDevice(prev_);
    }
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;
    int status() const { return status_; }

private:
    int prev_ = 0;
    int status_ = GQ_OK;
    bool switched_ = false;
};

struct TypeInfo {
    int unit_values;
    int unit_bytes;
    int block_values;   // 0 for float types
    bool asym;
};

bool type_info(int type, TypeInfo* ti) {
    switch (type) {
        case GQ_TYPE_F32: *ti = {1, 4, 0, false}; return true;
        case GQ_TYPE_F16: *ti = {1, 2, 0, false}; return true;
        case GQ_TYPE_BF16: *ti = {1, 2, 0, false}; return true;
        case GQ_TYPE_Q4_0: *ti = {32, 18, 32, false}; return true;
        case GQ_TYPE_Q8_0: *ti = {32, 34, 32, false}; return true;
        case GQ_TYPE_Q4_K: *ti = {256, 144, 32, true}; return true;
        case GQ_TYPE_Q5_K: *ti = {256, 176, 32, true}; return true;
        case GQ_TYPE_Q6_K: *ti = {256, 210, 16, false}; return true;
        case GQ_TYPE_Q4_1: *ti = {32, 20, 32, true}; return true;
        case GQ_TYPE_Q5_0: *ti = {32, 22, 32, false}; return true;
        case GQ_TYPE_Q5_1: *ti = {32, 24, 32, true}; return true;
        case GQ_TYPE_Q2_K: *ti = {256, 84, 16, true}; return true;
        case GQ_TYPE_Q3_K: *ti = {256, 110, 16, false}; return true;
        default: return false;
    }
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

bool valid_mask(int m) { return m == GQ_OUT_CODES || m == GQ_OUT_F32 || m == (GQ_OUT_CODES | GQ_OUT_F32); }

// Sizes, and the checks that need no pointers.
int shape_check(const gq_tensor_t& t, TypeInfo* ti, int64_t* n_values, int64_t* n_units) {
    if (!type_info(t.type, ti)) return GQ_ERR_TYPE;
    if (t.rows < 0 || t.cols < 0) return GQ_ERR_SIZE;
    if (t.cols != 0 && t.rows > INT64_MAX / t.cols) return GQ_ERR_SIZE;
    const int64_t nv = t.rows * t.cols;
    if (t.cols % ti->unit_values != 0) return GQ_ERR_SIZE;
    if (t.perm_heads < 0) return GQ_ERR_ARG;
    if (t.perm_heads > 0 && (t.rows % (2 * static_cast<int64_t>(t.perm_heads)) != 0)) return GQ_ERR_ARG;
    *n_values = nv;
    *n_units = nv / ti->unit_values;
    const int64_t need = *n_units * ti->unit_bytes;
    if (static_cast<uint64_t>(need) > t.src_bytes) return GQ_ERR_SIZE;
    return GQ_OK;
}

int validate(const gq_tensor_t& t, int out_mask, TypeInfo* ti, int64_t* n_values, int64_t* n_units) {
    const int st = shape_check(t, ti, n_values, n_units);
    if (st != GQ_OK) return st;
    if (*n_values == 0) return GQ_OK;
    if (t.src == nullptr) return GQ_ERR_NULL;
    if (!aligned(t.src, 16)) return GQ_ERR_ALIGN;
    if (ti->block_values == 0) {
        if (t.values == nullptr) return GQ_ERR_NULL;
        if (!aligned(t.values, 16)) return GQ_ERR_ALIGN;
        return GQ_OK;
    }
    if (out_mask & GQ_OUT_CODES) {
        if (t.codes == nullptr || t.scales == nullptr) return GQ_ERR_NULL;
        if (!aligned(t.codes, 16) || !aligned(t.scales, 4)) return GQ_ERR_ALIGN;
        if (t.diag != nullptr && !aligned(t.diag, 4)) return GQ_ERR_ALIGN;
    }
    if (out_mask & GQ_OUT_F32) {
        if (t.values == nullptr) return GQ_ERR_NULL;
        if (!aligned(t.values, 16)) return GQ_ERR_ALIGN;
    }
    return GQ_OK;
}

gq::GqDesc make_desc(const gq_tensor_t& t, const TypeInfo& ti, int64_t n_units) {
    gq::GqDesc d{};
    d.src = static_cast<const uint8_t*>(t.src);
    d.codes = static_cast<uint8_t*>(t.codes);
    d.scales = t.scales;
    d.values = t.values;
    d.diag = t.diag;
    d.n_units = n_units;
    d.units_per_row = t.cols / ti.unit_values;
    d.perm_heads = t.perm_heads;
    d.rows_per_head = t.perm_heads > 0 ? static_cast<int32_t>(t.rows / t.perm_heads) : 0;
    // unit indices of the tensor (plus a tile of slack) fit in 31 bits: 32-bit divisions
    if (t.perm_heads > 0 && n_units + 4096 < (int64_t(1) << 31)) {
        gq::fast_div_params(static_cast<uint32_t>(d.units_per_row), d.upr_mul, d.upr_shift);
        gq::fast_div_params(static_cast<uint32_t>(d.rows_per_head), d.rph_mul, d.rph_shift);
    }
    return d;
}

// Launch one kernel per GGML type present (the tensors are already validated).
int launch_grouped(const std::vector<std::pair<gq::GqDesc, int>>& items, int out_mask, void* stream) {
    static const int kTypes[] = {GQ_TYPE_Q4_K, GQ_TYPE_Q6_K, GQ_TYPE_Q5_K, GQ_TYPE_Q8_0, GQ_TYPE_Q4_0,
                                 GQ_TYPE_Q4_1, GQ_TYPE_Q5_0, GQ_TYPE_Q5_1, GQ_TYPE_Q2_K, GQ_TYPE_Q3_K,
                                 GQ_TYPE_F32, GQ_TYPE_F16, GQ_TYPE_BF16};
    std::unique_ptr<gq::GqBatch> b(new (std::nothrow) gq::GqBatch);
    if (!b) return GQ_ERR_NOMEM;
    for (int type : kTypes) {
        // F16 and BF16 are both 2-byte copies: launch them together
        if (type == GQ_TYPE_BF16) continue;
        auto same = [type](int t) { return t == type || (type == GQ_TYPE_F16 && t == GQ_TYPE_BF16); };
        b->n = 0;
        b->total_tiles = 0;
        for (size_t i = 0; i <= items.size(); ++i) {
            const bool last = i == items.size();
            if (!last && same(items[i].second)) {
                gq::GqDesc d = items[i].first;
                d.tile_begin = b->total_tiles;
                b->total_tiles += gq::tiles_for(type, d.n_units);
                b->d[b->n++] = d;
            }
            if ((last || b->n == gq::kMaxDesc) && b->n > 0) {
                const int e = gq::launch_batch(type, out_mask, *b, stream);
                if (e != 0) return cuda_status(e);
                b->n = 0;
                b->total_tiles = 0;
            }
        }
    }
    return GQ_OK;
}

}  // namespace

extern "C" {

int gq_version(void) { return GQ_ABI_VERSION; }

const char* gq_strerror(int status) {
    switch (status) {
        case GQ_OK: return "success";
        case GQ_ERR_TYPE: return "GGML type not supported by this path";
        case GQ_ERR_SIZE: return "sizes do not match the type's block geometry";
        case GQ_ERR_ALIGN: return "pointer not aligned as required";
        case GQ_ERR_NULL: return "a required pointer is NULL";
        case GQ_ERR_ARG: return "invalid argument";
        case GQ_ERR_CUDA: return "CUDA runtime error";
        case GQ_ERR_NOMEM: return "out of memory";
        default: return "unknown status";
    }
}

int gq_last_cuda_error(void) { return g_last_cuda; }

int gq_kernel_errors(int32_t device, int32_t clear, uint32_t* flags) {
    if (flags == nullptr) return GQ_ERR_NULL;
    *flags = 0;
    const DeviceScope scope(device);
    if (scope.status() != GQ_OK) return scope.status();
    return cuda_status(gq::kernel_errors(clear != 0, flags));
}

int gq_query(int32_t type, int64_t rows, int64_t cols, gq_layout_t* out) {
    if (out == nullptr) return GQ_ERR_NULL;
    gq_tensor_t t{};
    t.type = type;
    t.rows = rows;
    t.cols = cols;
    t.src_bytes = SIZE_MAX;
    TypeInfo ti;
    int64_t nv = 0, nu = 0;
    const int st = shape_check(t, &ti, &nv, &nu);
    if (st != GQ_OK) return st;
    out->n_values = nv;
    out->n_units = nu;
    out->src_bytes = nu * ti.unit_bytes;
    out->block_values = ti.block_values;
    out->unit_values = ti.unit_values;
    if (ti.block_values == 0) {
        out->codes_bytes = 0;
        out->scales_count = 0;
        out->values_bytes = nv * ti.unit_bytes;
    } else {
        out->codes_bytes = nv;
        out->scales_count = nv / ti.block_values;
        out->values_bytes = 4 * nv;
    }
    return GQ_OK;
}

int gq_diag_reset(gq_diag_t* diag, int32_t count, void* stream) {
    if (count < 0) return GQ_ERR_ARG;
    if (count == 0) return GQ_OK;
    if (diag == nullptr) return GQ_ERR_NULL;
    return cuda_status(cudaMemsetAsync(diag, 0, sizeof(gq_diag_t) * count, static_cast<cudaStream_t>(stream)));
}

int gq_convert_batch(const gq_tensor_t* tensors, int32_t count, int32_t out_mask, void* stream) {
    if (count < 0) return GQ_ERR_ARG;
    if (count > 0 && tensors == nullptr) return GQ_ERR_NULL;
    if (!valid_mask(out_mask)) return GQ_ERR_ARG;
    std::vector<std::pair<gq::GqDesc, int>> items;
    items.reserve(count);
    for (int i = 0; i < count; ++i) {
        TypeInfo ti;
        int64_t nv = 0, nu = 0;
        const int st = validate(tensors[i], out_mask, &ti, &nv, &nu);
        if (st != GQ_OK) return st;
        if (nv == 0) continue;
        items.emplace_back(make_desc(tensors[i], ti, nu), tensors[i].type);
    }
    return launch_grouped(items, out_mask, stream);
}

int gq_convert(const gq_tensor_t* tensor, int32_t out_mask, void* stream) {
    if (tensor == nullptr) return GQ_ERR_NULL;
    if (!valid_mask(out_mask)) return GQ_ERR_ARG;
    TypeInfo ti;
    int64_t nv = 0, nu = 0;
    const int st = validate(*tensor, out_mask, &ti, &nv, &nu);
    if (st != GQ_OK) return st;
    if (tensor->diag != nullptr && ti.asym && (out_mask & GQ_OUT_CODES)) {
        const int e = gq_diag_reset(tensor->diag, 1, stream);
        if (e != GQ_OK) return e;
    }
    return gq_convert_batch(tensor, 1, out_mask, stream);
}

int gq_requantize_symmetric(const float* block_consts, const int8_t* codes, int64_t n_blocks,
                            int32_t block, int32_t output_bits, float* out_scales,
                            int8_t* out_codes, gq_diag_t* diag, void* stream) {
    if (n_blocks < 0 || block < 1 || block > 256 || output_bits < 2 || output_bits > 8) return GQ_ERR_ARG;
    if (diag != nullptr) {
        const int e = gq_diag_reset(diag, 1, stream);
        if (e != GQ_OK) return e;
    }
    if (n_blocks == 0) return GQ_OK;
    if (!block_consts || !codes || !out_scales || !out_codes) return GQ_ERR_NULL;
    if (!aligned(block_consts, 4) || !aligned(out_scales, 4)) return GQ_ERR_ALIGN;
    return cuda_status(gq::launch_requant(block_consts, codes, n_blocks, block, output_bits, out_scales,
                                          out_codes, diag, stream));
}

}  // extern "C"

namespace {

// Checks of one tensor for the fused layout writer and its descriptor (tile_begin 0).
// Returns GQ_OK with *empty set when there is nothing to launch.
int modalix_desc(const gq_tensor_t& t, int64_t rows_padded, gq::GqModalix* m, bool* empty) {
    TypeInfo ti;
    int64_t nv = 0, nu = 0;
    const int st = shape_check(t, &ti, &nv, &nu);
    if (st != GQ_OK) return st;
    if (ti.block_values == 0) return GQ_ERR_TYPE;
    if (rows_padded < t.rows || rows_padded > INT32_MAX) return GQ_ERR_SIZE;
    // whole 256-channel column tiles, and every row's bytes starting on a 16-byte boundary
    if (t.cols % gq::kModalixCols != 0) return GQ_ERR_SIZE;
    const int64_t upr = t.cols / ti.unit_values;
    if ((upr * ti.unit_bytes) % 16 != 0) return GQ_ERR_SIZE;
    *empty = t.cols == 0 || rows_padded == 0;
    if (*empty) return GQ_OK;
    if (t.codes == nullptr || t.scales == nullptr) return GQ_ERR_NULL;
    if (t.rows > 0 && t.src == nullptr) return GQ_ERR_NULL;
    if (!aligned(t.src, 16) || !aligned(t.scales, 4)) return GQ_ERR_ALIGN;
    if (t.diag != nullptr && !aligned(t.diag, 4)) return GQ_ERR_ALIGN;
    const int64_t n_col = t.cols / gq::kModalixCols;
    const int64_t n_tiles = (rows_padded + gq::kModalixRows - 1) / gq::kModalixRows * n_col;
    if (n_tiles >= (int64_t(1) << 31)) return GQ_ERR_SIZE;
    *m = gq::GqModalix{};
    m->src = static_cast<const uint8_t*>(t.src);
    m->out_codes = static_cast<uint8_t*>(t.codes);
    m->out_scales = t.scales;
    m->diag = (ti.asym && t.diag != nullptr) ? t.diag : nullptr;
    m->rows = t.rows;
    m->cols = t.cols;
    m->rows_padded = rows_padded;
    m->units_per_row = upr;
    m->n_col_tiles = static_cast<uint32_t>(n_col);
    m->n_tiles = static_cast<uint32_t>(n_tiles);
    gq::fast_div_params(m->n_col_tiles, m->ncol_mul, m->ncol_shift);
    m->head_dim = t.perm_heads > 0 ? static_cast<int32_t>(t.rows / t.perm_heads) : 0;
    return GQ_OK;
}

}  // namespace

extern "C" {

int gq_convert_modalix_batch(const gq_tensor_t* tensors, const int64_t* rows_padded, int32_t count,
                             void* stream) {
    if (count < 0) return GQ_ERR_ARG;
    if (count > 0 && tensors == nullptr) return GQ_ERR_NULL;
    std::vector<std::pair<gq::GqModalix, int>> items;
    items.reserve(count);
    for (int i = 0; i < count; ++i) {
        const gq_tensor_t& t = tensors[i];
        gq::GqModalix m;
        bool empty = false;
        const int st = modalix_desc(t, rows_padded ? rows_padded[i] : t.rows, &m, &empty);
        if (st != GQ_OK) return st;
        if (t.diag != nullptr) {
            const int e = gq_diag_reset(t.diag, 1, stream);
            if (e != GQ_OK) return e;
        }
        if (!empty) items.emplace_back(m, t.type);
    }
    static const int kTypes[] = {GQ_TYPE_Q4_K, GQ_TYPE_Q6_K, GQ_TYPE_Q5_K, GQ_TYPE_Q8_0, GQ_TYPE_Q4_0,
                                 GQ_TYPE_Q4_1, GQ_TYPE_Q5_0, GQ_TYPE_Q5_1, GQ_TYPE_Q2_K, GQ_TYPE_Q3_K};
    std::unique_ptr<gq::GqModalixBatch> b(new (std::nothrow) gq::GqModalixBatch);
    if (!b) return GQ_ERR_NOMEM;
    for (int type : kTypes) {
        b->n = 0;
        b->total_tiles = 0;
        for (size_t i = 0; i <= items.size(); ++i) {
            const bool last = i == items.size();
            if (!last && items[i].second == type) {
                if (static_cast<uint64_t>(b->total_tiles) + items[i].first.n_tiles >= (uint64_t(1) << 31)) {
                    const int e = cuda_status(gq::launch_modalix(type, *b, stream));
                    if (e != GQ_OK) return e;
                    b->n = 0;
                    b->total_tiles = 0;
                }
                gq::GqModalix m = items[i].first;
                m.tile_begin = b->total_tiles;
                b->total_tiles += m.n_tiles;
                b->d[b->n++] = m;
            }
            if ((last || b->n == gq::kMaxModalix) && b->n > 0) {
                const int e = cuda_status(gq::launch_modalix(type, *b, stream));
                if (e != GQ_OK) return e;
                b->n = 0;
                b->total_tiles = 0;
            }
        }
    }
    return GQ_OK;
}

int gq_convert_modalix(const gq_tensor_t* tensor, int64_t rows_padded, void* stream) {
    if (tensor == nullptr) return GQ_ERR_NULL;
    return gq_convert_modalix_batch(tensor, &rows_padded, 1, stream);
}

int gq_unpack_fields(int32_t type, const void* src, size_t src_bytes, int64_t n_units, float* super_consts,
                     int8_t* block_consts, int8_t* values, void* stream) {
    TypeInfo ti;
    if (!type_info(type, &ti)) return GQ_ERR_TYPE;
    const bool kq = ti.unit_values == 256;
    if (!kq && type != GQ_TYPE_Q4_1 && type != GQ_TYPE_Q5_1) return GQ_ERR_TYPE;
    if (n_units < 0 || n_units > INT64_MAX / 256) return GQ_ERR_SIZE;
    if (static_cast<uint64_t>(n_units) * ti.unit_bytes > src_bytes) return GQ_ERR_SIZE;
    if (n_units == 0) return GQ_OK;
    if (src == nullptr || super_consts == nullptr || values == nullptr) return GQ_ERR_NULL;
    if (kq != (block_consts != nullptr)) return block_consts ? GQ_ERR_ARG : GQ_ERR_NULL;
    if (!aligned(src, 16) || !aligned(values, 16) || !aligned(super_consts, 8) ||
        (block_consts && !aligned(block_consts, 8)))
        return GQ_ERR_ALIGN;
    return cuda_status(gq::launch_fields(type, static_cast<const uint8_t*>(src), n_units, super_consts,
                                         block_consts, values, stream));
}

int gq_remove_superblocks(const float* super_consts, const void* block_consts, int32_t block_elem_bytes,
                          int64_t n_super, int32_t blocks_per_super, int32_t n_consts, uint16_t* out_f16,
                          float* out_f32, void* stream) {
    if (block_elem_bytes != 1 && block_elem_bytes != 2) return GQ_ERR_ARG;
    if (n_consts != 1 && n_consts != 2) return GQ_ERR_ARG;
    if (n_super < 0 || blocks_per_super < 1 || n_super > INT64_MAX / (2 * int64_t(blocks_per_super)))
        return GQ_ERR_SIZE;
    if (n_super == 0) return GQ_OK;
    if (super_consts == nullptr || block_consts == nullptr || (out_f16 == nullptr && out_f32 == nullptr))
        return GQ_ERR_NULL;
    if (!aligned(super_consts, 4) || !aligned(block_consts, block_elem_bytes) || !aligned(out_f16, 2) ||
        !aligned(out_f32, 4))
        return GQ_ERR_ALIGN;
    return cuda_status(gq::launch_superblocks(super_consts, block_consts, block_elem_bytes, n_super,
                                              blocks_per_super, n_consts, out_f16, out_f32, stream));
}

int gq_modalix_layout(const void* codes, const float* scales, int64_t rows, int64_t cols, int32_t block_values,
                      int64_t rows_padded, void* out_codes, float* out_scales, void* stream) {
    if (rows < 0 || cols < 0 || rows_padded < rows) return GQ_ERR_SIZE;
    if (block_values <= 0 || cols % block_values != 0) return GQ_ERR_SIZE;
    if (cols > (int64_t(65535) * 32) || rows_padded > INT32_MAX) return GQ_ERR_SIZE;
    if (rows_padded == 0 || cols == 0) return GQ_OK;
    if ((codes == nullptr) != (out_codes == nullptr) || (scales == nullptr) != (out_scales == nullptr))
        return GQ_ERR_NULL;
    if (codes == nullptr && scales == nullptr) return GQ_ERR_NULL;
    if ((scales && !aligned(scales, 4)) || (out_scales && !aligned(out_scales, 4))) return GQ_ERR_ALIGN;
    return cuda_status(gq::launch_layout(static_cast<const uint8_t*>(codes), scales, rows, cols, cols / block_values,
                                         rows_padded, static_cast<uint8_t*>(out_codes), out_scales, stream));
}

int gq_embedding_rows(int32_t type, const void* src, size_t src_bytes, int64_t rows, int64_t cols,
                      float embed_scale, int32_t quantize, int8_t* codes, uint16_t* scales_bf16, float* values,
                      void* stream) {
    TypeInfo ti;
    if (!type_info(type, &ti)) return GQ_ERR_TYPE;
    switch (type) {   // the formats token embeddings come in
        case GQ_TYPE_F32: case GQ_TYPE_F16: case GQ_TYPE_BF16: case GQ_TYPE_Q8_0: case GQ_TYPE_Q4_0:
        case GQ_TYPE_Q4_K: case GQ_TYPE_Q5_K: case GQ_TYPE_Q6_K: break;
        default: return GQ_ERR_TYPE;
    }
    if (rows < 0 || cols < 0 || cols % ti.unit_values != 0 || cols % 4 != 0) return GQ_ERR_SIZE;
    const int64_t row_bytes = cols / ti.unit_values * ti.unit_bytes;
    if (row_bytes > gq::embed_max_row_bytes()) return GQ_ERR_SIZE;
    if (cols != 0 && rows > INT64_MAX / cols) return GQ_ERR_SIZE;
    if (static_cast<uint64_t>(rows * row_bytes) > src_bytes) return GQ_ERR_SIZE;
    if (rows == 0 || cols == 0) return GQ_OK;
    if (src == nullptr) return GQ_ERR_NULL;
    if (!aligned(src, 16)) return GQ_ERR_ALIGN;
    if (quantize) {
        if (codes == nullptr || scales_bf16 == nullptr) return GQ_ERR_NULL;
        if (!aligned(codes, 4) || !aligned(scales_bf16, 2)) return GQ_ERR_ALIGN;
    } else {
        if (values == nullptr) return GQ_ERR_NULL;
        if (!aligned(values, 16)) return GQ_ERR_ALIGN;
    }
    return cuda_status(gq::launch_embed(type, false, static_cast<const uint8_t*>(src), rows, cols, row_bytes,
                                        embed_scale, quantize ? 1 : 0, codes, scales_bf16, values,
                                        static_cast<int64_t>(src_bytes), stream));
}

int gq_quantize_rows(const float* x, int64_t rows, int64_t cols, int8_t* codes, uint16_t* scales_bf16,
                     void* stream) {
    if (rows < 0 || cols < 0 || cols % 4 != 0) return GQ_ERR_SIZE;
    if (cols * 4 > gq::embed_max_row_bytes()) return GQ_ERR_SIZE;
    if (rows == 0 || cols == 0) return GQ_OK;
    if (x == nullptr || codes == nullptr || scales_bf16 == nullptr) return GQ_ERR_NULL;
    if (!aligned(x, 16) || !aligned(codes, 4) || !aligned(scales_bf16, 2)) return GQ_ERR_ALIGN;
    return cuda_status(gq::launch_embed(GQ_TYPE_F32, true, reinterpret_cast<const uint8_t*>(x), rows, cols, cols * 4,
                                        1.0f, 1, codes, scales_bf16, nullptr, rows * cols * 4, stream));
}

// ---------------------------------------------------------------------------------------
// Page-locked result buffers, recycled
//
// The drop-in call returns a fresh array per tensor.  A fresh pageable array costs the
// kernel's page zeroing on first touch and a host copy out of a pinned bounce slot; a
// page-locked one is written by the copy engines directly.  Buffers are handed out in size
// classes (two per octave) and a released buffer waits for the next request of its class,
// so a caller that converts one tensor at a time pays for pinning once per class.
// ---------------------------------------------------------------------------------------

namespace {

struct HostArena {
    std::mutex mu;
    pid_t pid = 0;
    size_t limit = 0;      // in use + cached, bytes
    size_t in_use = 0;
    size_t cached = 0;
    std::map<size_t, std::vector<void*>> free_by_class;
    struct Block {
        size_t bytes;
        bool mapped;   // anonymous map + cudaHostRegister (else cudaHostAlloc)
    };
    std::unordered_map<void*, Block> owned;   // every block of this process

    void init_locked() {
        if (pid == getpid()) return;
        // a forked child owns none of its parent's page-locked blocks
        pid = getpid();
        in_use = cached = 0;
        free_by_class.clear();
        owned.clear();
        long mb = -1;
        if (const char* e = std::getenv("LLIMA_B200_PINNED_RESULTS_MB")) mb = std::atol(e);
        if (mb >= 0) {
            limit = static_cast<size_t>(mb) << 20;
        } else {
            const long pages = sysconf(_SC_PHYS_PAGES), page = sysconf(_SC_PAGE_SIZE);
            const size_t phys = (pages > 0 && page > 0) ? static_cast<size_t>(pages) * static_cast<size_t>(page) : 0;
            limit = std::min<size_t>(phys / 4, size_t(16) << 30);
        }
    }
};
HostArena g_arena;

// A new page-locked block.  From 2 MiB on: anonymous memory with transparent huge pages
// requested, then registered with CUDA (pinning 2 MiB pages costs far less than the 4 KiB
// pages cudaHostAlloc pins); cudaHostAlloc below that or where registration fails.
void* arena_block(size_t bytes, bool* mapped) {
    if (bytes >= (size_t(2) << 20)) {
        void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
        if (p != MAP_FAILED) {
            madvise(p, bytes, MADV_HUGEPAGE);
            if (cudaHostRegister(p, bytes, cudaHostRegisterPortable) == cudaSuccess) {
                *mapped = true;
                return p;
            }
            cudaGetLastError();
            munmap(p, bytes);
        }
    }
    void* q = nullptr;
    if (cudaHostAlloc(&q, bytes, cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    *mapped = false;
    return q;
}

void arena_release(void* p, const HostArena::Block& b) {
    if (b.mapped) {
        cudaHostUnregister(p);
        munmap(p, b.bytes);
    } else {
        cudaFreeHost(p);
    }
}

// Smallest size class >= bytes: 2^k or 3 * 2^(k-1), at least 64 KiB.
size_t size_class(size_t bytes) {
    size_t c = size_t(64) << 10;
    while (c < bytes) {
        const size_t mid = c + c / 2;
        if (mid >= bytes) return mid;
        c *= 2;
    }
    return c;
}

}  // namespace

extern "C" {

int gq_host_alloc(size_t bytes, void** out) {
    if (out == nullptr) return GQ_ERR_NULL;
    *out = nullptr;
    if (bytes == 0) return GQ_ERR_ARG;
    const size_t cls = size_class(bytes);
    std::lock_guard<std::mutex> lock(g_arena.mu);
    g_arena.init_locked();
    auto it = g_arena.free_by_class.find(cls);
    if (it != g_arena.free_by_class.end() && !it->second.empty()) {
        *out = it->second.back();
        it->second.pop_back();
        g_arena.cached -= cls;
        g_arena.in_use += cls;
        return GQ_OK;
    }
    // make room: release cached blocks of other classes first
    while (g_arena.in_use + g_arena.cached + cls > g_arena.limit && g_arena.cached > 0) {
        auto big = std::prev(g_arena.free_by_class.end());
        while (big->second.empty()) big = std::prev(big);
        void* victim = big->second.back();
        arena_release(victim, g_arena.owned[victim]);
        g_arena.owned.erase(victim);
        big->second.pop_back();
        g_arena.cached -= big->first;
    }
    if (g_arena.in_use + cls > g_arena.limit) return GQ_ERR_NOMEM;
    bool mapped = false;
    void* p = arena_block(cls, &mapped);
    if (p == nullptr) return GQ_ERR_NOMEM;
    g_arena.owned[p] = HostArena::Block{cls, mapped};
    g_arena.in_use += cls;
    *out = p;
    return GQ_OK;
}

int gq_host_free(void* p) {
    if (p == nullptr) return GQ_OK;
    std::lock_guard<std::mutex> lock(g_arena.mu);
    if (g_arena.pid != getpid()) return GQ_ERR_ARG;   // not from this process's arena
    auto it = g_arena.owned.find(p);
    if (it == g_arena.owned.end()) return GQ_ERR_ARG;
    const size_t cls = it->second.bytes;
    g_arena.in_use -= cls;
    g_arena.free_by_class[cls].push_back(p);
    g_arena.cached += cls;
    return GQ_OK;
}

int gq_host_trim(void) {
    std::lock_guard<std::mutex> lock(g_arena.mu);
    if (g_arena.pid != getpid()) return GQ_OK;
    for (auto& kv : g_arena.free_by_class) {
        for (void* p : kv.second) {
            arena_release(p, g_arena.owned[p]);
            g_arena.owned.erase(p);
        }
        kv.second.clear();
    }
    g_arena.cached = 0;
    return GQ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Host-buffer session
//
// A request is cut into pieces of about piece_target() bytes of device footprint (input +
// outputs; a permuted tensor stays whole), and the pieces rotate through kSlots device
// slots, each with its own stream.  Pinned host buffers are copied by the DMA engines
// directly.  A pageable one (a numpy array, the memory map of a GGUF file) is bounced
// through a pinned host slot laid out like the device slot: a pool of host threads copies
// the piece's input into it, the GPU copies it in, converts and copies the results back to
// it, and the pool copies them to the caller's buffers.  While the GPU works on piece p the
// host drains piece p - 1 and fills piece p + 1, so the host copies, both PCIe directions
// and the kernels overlap, within one tensor as well as across tensors.
// ---------------------------------------------------------------------------------------

namespace {

constexpr int kSlots = 3;
constexpr size_t kPieceTargetDefault = size_t(64) << 20;

// Slot footprint of one piece (LLIMA_B200_PIECE_MB overrides; at least 1 MiB).
size_t piece_target() {
    static const size_t v = [] {
        if (const char* e = std::getenv("LLIMA_B200_PIECE_MB")) {
            const long mb = std::atol(e);
            if (mb >= 1) return static_cast<size_t>(mb) << 20;
        }
        return kPieceTargetDefault;
    }();
    return v;
}
constexpr size_t kCopyChunk = size_t(2) << 20;

struct CopyJob {
    void* dst;
    const void* src;
    size_t bytes;
};

// Host threads that split a list of copies into chunks and run them together with the
// calling thread.  Pageable destinations are first touched here, so their page faults
// are taken in parallel too.
class CopyPool {
  public:
    explicit CopyPool(int threads) {
        for (int i = 1; i < threads; ++i) workers_.emplace_back([this] { work(); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> g(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }
    void run(const std::vector<CopyJob>& jobs) {
        auto b = std::make_shared<Batch>();
        for (const CopyJob& j : jobs)
            for (size_t o = 0; o < j.bytes; o += kCopyChunk)
                b->chunks.push_back({static_cast<uint8_t*>(j.dst) + o, static_cast<const uint8_t*>(j.src) + o,
                                     std::min(kCopyChunk, j.bytes - o)});
        if (b->chunks.empty()) return;
        b->left.store(b->chunks.size());
        if (!workers_.empty() && b->chunks.size() > 1) {
            {
                std::lock_guard<std::mutex> g(mu_);
                current_ = b;
                ++gen_;
            }
            cv_.notify_all();
        }
        copy(*b);
        std::unique_lock<std::mutex> g(b->mu);
        b->cv.wait(g, [&] { return b->left.load() == 0; });
    }

  private:
    struct Batch {
        std::vector<CopyJob> chunks;
        std::atomic<size_t> next{0};
        std::atomic<size_t> left{0};
        std::mutex mu;
        std::condition_variable cv;
    };
    static void copy(Batch& b) {
        for (;;) {
            const size_t i = b.next.fetch_add(1);
            if (i >= b.chunks.size()) return;
            std::memcpy(b.chunks[i].dst, b.chunks[i].src, b.chunks[i].bytes);
            if (b.left.fetch_sub(1) == 1) {
                std::lock_guard<std::mutex> g(b.mu);
                b.cv.notify_all();
            }
        }
    }
    void work() {
        uint64_t seen = 0;
        for (;;) {
            std::shared_ptr<Batch> b;
            {
                std::unique_lock<std::mutex> g(mu_);
                cv_.wait(g, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
                b = current_;
            }
            if (b) copy(*b);
        }
    }
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::shared_ptr<Batch> current_;
    uint64_t gen_ = 0;
    bool stop_ = false;
};

// Background threads that fault in the pages of pageable result buffers ahead of the copies
// that fill them (madvise MADV_POPULATE_WRITE: the kernel maps and zeroes the pages, and
// never changes the content of a page that is already there, so it can run beside the
// copies).  Fresh result arrays otherwise take one page fault per page inside those copies,
// which bounds the host side of a pageable request.  Kernels without the advice (before
// Linux 5.14) refuse it and nothing is done.
class PrefaultPool {
  public:
    explicit PrefaultPool(int threads) {
        for (int i = 0; i < threads; ++i) workers_.emplace_back([this] { work(); });
    }
    ~PrefaultPool() {
        {
            std::lock_guard<std::mutex> g(mu_);
            stop_ = true;
            q_.clear();
        }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }
    // Queue [p, p + bytes) (whole pages inside it), in order.
    void submit(void* p, size_t bytes) {
        const uintptr_t page = static_cast<uintptr_t>(sysconf(_SC_PAGESIZE));
        uintptr_t a = (reinterpret_cast<uintptr_t>(p) + page - 1) & ~(page - 1);
        const uintptr_t end = (reinterpret_cast<uintptr_t>(p) + bytes) & ~(page - 1);
        std::lock_guard<std::mutex> g(mu_);
        if (stop_ || unsupported_.load()) return;
        for (; a < end; a += kChunk) q_.push_back({a, std::min<uintptr_t>(kChunk, end - a)});
        cv_.notify_all();
    }
    // Drop what has not started and wait for what has (the buffers may be freed next).
    void cancel() {
        std::unique_lock<std::mutex> g(mu_);
        q_.clear();
        idle_.wait(g, [&] { return active_ == 0; });
    }

  private:
    static constexpr uintptr_t kChunk = uintptr_t(8) << 20;
    struct Range {
        uintptr_t a, n;
    };
    void work() {
        for (;;) {
            Range r;
            {
                std::unique_lock<std::mutex> g(mu_);
                cv_.wait(g, [&] { return stop_ || !q_.empty(); });
                if (stop_) return;
                r = q_.front();
                q_.pop_front();
                ++active_;
            }
#ifdef MADV_POPULATE_WRITE
            if (madvise(reinterpret_cast<void*>(r.a), r.n, MADV_POPULATE_WRITE) != 0 && errno == EINVAL)
                unsupported_.store(true);
#endif
            {
                std::lock_guard<std::mutex> g(mu_);
                --active_;
            }
            idle_.notify_all();
        }
    }
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_, idle_;
    std::deque<Range> q_;
    int active_ = 0;
    bool stop_ = false;
    std::atomic<bool> unsupported_{false};
};

int copy_threads() {
    if (const char* e = std::getenv("LLIMA_B200_COPY_THREADS")) {
        const int n = std::atoi(e);
        if (n >= 1) return std::min(n, 64);
    }
    const int hw = static_cast<int>(std::thread::hardware_concurrency());
    return std::max(1, std::min(8, hw / 2));
}

// A host pointer the DMA engines cannot read or write directly (not pinned or registered).
bool pageable(const void* p) {
    if (p == nullptr) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return true;
    }
    return a.type != cudaMemoryTypeHost && a.type != cudaMemoryTypeManaged;
}

}  // namespace

struct gq_session {
    int device = 0;
    size_t slot_bytes = 0;
    uint8_t* slot[kSlots] = {};
    uint8_t* pinned[kSlots] = {};   // host bounce slots, allocated on first pageable use
    bool pinned_failed = false;
    cudaStream_t stream[kSlots] = {};
    cudaEvent_t done[kSlots] = {};
    gq_diag_t* d_diag = nullptr;
    int diag_cap = 0;
    std::unique_ptr<CopyPool> pool;
    std::unique_ptr<PrefaultPool> prefault;
    std::mutex mu;                  // one gq_convert_host at a time per session
};

namespace {

// After a call's work has finished: GQ_OK, or GQ_ERR_CUDA (cudaErrorTimeout) when a
// conversion kernel on the current device gave up waiting for a copy (flags cleared).
int kernels_ok() {
    uint32_t flags = 0;
    const int e = gq::kernel_errors(true, &flags);
    if (e != 0) return cuda_status(e);
    return flags != 0 ? cuda_status(cudaErrorTimeout) : GQ_OK;
}

constexpr size_t kAlign = 256;
size_t round_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

// Device bytes one unit of a tensor occupies in a staging slot.
size_t unit_footprint(const TypeInfo& ti, int out_mask) {
    size_t b = ti.unit_bytes;
    if (ti.block_values == 0) return b + ti.unit_bytes;
    if (out_mask & GQ_OUT_CODES) b += ti.unit_values + 4 * (ti.unit_values / ti.block_values);
    if (out_mask & GQ_OUT_F32) b += 4 * static_cast<size_t>(ti.unit_values);
    return b;
}

struct Member {
    int tensor;
    int64_t unit0;
    int64_t units;
};


// Pinned bounce slots and the copy pool, on the first request with a pageable buffer.
// Without them (pinned allocation refused) pageable buffers are handed to the copy
// engines as they are.
bool ensure_bounce(gq_session* s) {
    if (s->pinned[0] != nullptr) return true;
    if (s->pinned_failed) return false;
    for (int k = 0; k < kSlots; ++k) {
        if (cudaHostAlloc(reinterpret_cast<void**>(&s->pinned[k]), s->slot_bytes, cudaHostAllocDefault) !=
            cudaSuccess) {
            cudaGetLastError();
            for (int j = 0; j < kSlots; ++j) {
                if (s->pinned[j]) cudaFreeHost(s->pinned[j]);
                s->pinned[j] = nullptr;
            }
            s->pinned_failed = true;
            return false;
        }
    }
    if (!s->pool) s->pool.reset(new (std::nothrow) CopyPool(copy_threads()));
    if (!s->prefault) s->prefault.reset(new (std::nothrow) PrefaultPool(std::max(1, copy_threads() / 2)));
    return s->pool != nullptr && s->prefault != nullptr;
}

}  // namespace

int gq_session_create(int32_t device, size_t staging_bytes, gq_session_t** out) {
    if (out == nullptr) return GQ_ERR_NULL;
    *out = nullptr;
    if (staging_bytes < (1u << 20)) return GQ_ERR_ARG;
    const DeviceScope scope(device);
    if (scope.status() != GQ_OK) return scope.status();
    std::unique_ptr<gq_session> s(new (std::nothrow) gq_session);
    if (!s) return GQ_ERR_NOMEM;
    s->device = device;
    s->slot_bytes = staging_bytes & ~(kAlign - 1);
    for (int i = 0; i < kSlots; ++i) {
        if (cudaMalloc(&s->slot[i], s->slot_bytes) != cudaSuccess) {
            gq_session_destroy(s.release());
            cudaGetLastError();
            return GQ_ERR_NOMEM;
        }
        if (cudaStreamCreateWithFlags(&s->stream[i], cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&s->done[i], cudaEventDisableTiming) != cudaSuccess) {
            const int e = cuda_status(cudaGetLastError());
            gq_session_destroy(s.release());
            return e;
        }
    }
    *out = s.release();
    return GQ_OK;
}

int gq_session_destroy(gq_session_t* s) {
    if (s == nullptr) return GQ_OK;
    const DeviceScope scope(s->device);
    for (int i = 0; i < kSlots; ++i) {
        if (s->stream[i]) cudaStreamSynchronize(s->stream[i]);
    }
    s->pool.reset();
    s->prefault.reset();
    for (int i = 0; i < kSlots; ++i) {
        if (s->done[i]) cudaEventDestroy(s->done[i]);
        if (s->stream[i]) cudaStreamDestroy(s->stream[i]);
        if (s->slot[i]) cudaFree(s->slot[i]);
        if (s->pinned[i]) cudaFreeHost(s->pinned[i]);
    }
    if (s->d_diag) cudaFree(s->d_diag);
    delete s;
    return GQ_OK;
}

int gq_convert_host(gq_session_t* s, const gq_tensor_t* tensors, int32_t count, int32_t out_mask,
                    gq_diag_t* host_diags) {
    if (s == nullptr) return GQ_ERR_NULL;
    if (count < 0) return GQ_ERR_ARG;
    if (count > 0 && tensors == nullptr) return GQ_ERR_NULL;
    if (!valid_mask(out_mask)) return GQ_ERR_ARG;
    std::lock_guard<std::mutex> session_lock(s->mu);
    const DeviceScope scope(s->device);
    int st = scope.status();
    if (st != GQ_OK) return st;

    std::vector<TypeInfo> info(count);
    std::vector<int64_t> units(count);
    std::vector<uint8_t> bounce_in(count, 0), bounce_out(count, 0);
    bool any_bounce = false;
    for (int i = 0; i < count; ++i) {
        int64_t nv = 0;
        // host pointers: alignment of the host copy source does not matter
        const gq_tensor_t& t = tensors[i];
        st = shape_check(t, &info[i], &nv, &units[i]);
        if (st != GQ_OK) return st;
        if (nv == 0) continue;
        if (t.src == nullptr) return GQ_ERR_NULL;
        if (info[i].block_values == 0) {
            if (t.values == nullptr) return GQ_ERR_NULL;
        } else {
            if ((out_mask & GQ_OUT_CODES) && (t.codes == nullptr || t.scales == nullptr)) return GQ_ERR_NULL;
            if ((out_mask & GQ_OUT_F32) && t.values == nullptr) return GQ_ERR_NULL;
        }
        // a permuted tensor is cut into whole heads (the permutation keeps them apart): one
        // head must fit a slot
        if (t.perm_heads > 0 &&
            round_up((t.rows / t.perm_heads) * (t.cols / info[i].unit_values) * unit_footprint(info[i], out_mask)) +
                    4 * kAlign > s->slot_bytes)
            return GQ_ERR_SIZE;
        bounce_in[i] = pageable(t.src);
        if (info[i].block_values == 0) {
            bounce_out[i] = pageable(t.values);
        } else {
            bounce_out[i] = ((out_mask & GQ_OUT_CODES) && (pageable(t.codes) || pageable(t.scales))) ||
                            ((out_mask & GQ_OUT_F32) && pageable(t.values));
        }
        any_bounce |= bounce_in[i] || bounce_out[i];
    }
    if (any_bounce && !ensure_bounce(s)) {
        std::fill(bounce_in.begin(), bounce_in.end(), 0);
        std::fill(bounce_out.begin(), bounce_out.end(), 0);
    }

    // on an error after work was queued, let the queued work finish before returning, so
    // that nothing still writes into the slots or the caller's buffers
    auto fail = [&](int e) {
        for (int k = 0; k < kSlots; ++k) cudaStreamSynchronize(s->stream[k]);
        cudaGetLastError();
        if (s->prefault) s->prefault->cancel();
        return e;
    };

    if (host_diags != nullptr && count > s->diag_cap) {
        if (s->d_diag) cudaFree(s->d_diag);
        s->d_diag = nullptr;
        s->diag_cap = 0;
        if (cudaMalloc(&s->d_diag, sizeof(gq_diag_t) * count) != cudaSuccess) {
            cudaGetLastError();
            return GQ_ERR_NOMEM;
        }
        s->diag_cap = count;
    }
    if (host_diags != nullptr && count > 0) {
        st = cuda_status(cudaMemsetAsync(s->d_diag, 0, sizeof(gq_diag_t) * count, s->stream[0]));
        if (st != GQ_OK) return st;
        // the other streams must not run their kernels before the zeroing
        if ((st = cuda_status(cudaEventRecord(s->done[0], s->stream[0]))) != GQ_OK) return fail(st);
        for (int k = 1; k < kSlots; ++k) cudaStreamWaitEvent(s->stream[k], s->done[0], 0);
    }

    // Cut the work into pieces of about piece_target() bytes of slot footprint: large
    // tensors are split on unit boundaries (permuted ones on head boundaries), small ones
    // are packed together.
    // A small request is cut into at least two pieces, so that its host copies, both copy
    // directions and the kernels still overlap (whole models use the full piece size;
    // measured on the per-tensor calls of the 8B set: halves 12.4, quarters 11.1, eighths
    // 11.7 GB/s).
    size_t request = 0;
    for (int i = 0; i < count; ++i) request += static_cast<size_t>(units[i]) * unit_footprint(info[i], out_mask);
    const size_t target = std::min({s->slot_bytes, piece_target(), std::max(size_t(4) << 20, request / 2)});
    std::vector<std::vector<Member>> pieces;
    {
        std::vector<Member> cur;
        size_t used = 0;
        for (int i = 0; i < count; ++i) {
            int64_t done = 0;
            const size_t fp = unit_footprint(info[i], out_mask);
            const gq_tensor_t& t = tensors[i];
            // pieces of a permuted tensor hold whole heads
            const int64_t step = t.perm_heads > 0 ? (t.rows / t.perm_heads) * (t.cols / info[i].unit_values) : 1;
            while (done < units[i]) {
                const size_t room = target > used + 4 * kAlign ? target - used - 4 * kAlign : 0;
                int64_t take = static_cast<int64_t>(room / fp) / step * step;
                if (take <= 0) {
                    if (cur.empty()) {
                        // one step larger than the piece target still fits a slot (checked above)
                        take = step;
                        if (round_up(step * fp) + 4 * kAlign > s->slot_bytes) return fail(GQ_ERR_SIZE);
                    } else {
                        pieces.push_back(std::move(cur));
                        cur.clear();
                        used = 0;
                        continue;
                    }
                }
                take = std::min<int64_t>(take, units[i] - done);
                cur.push_back({i, done, take});
                used += round_up(take * fp) + 4 * kAlign;
                done += take;
            }
        }
        if (!cur.empty()) pieces.push_back(std::move(cur));
    }

    // pageable result buffers: fault their pages in ahead of the copies, piece by piece
    if (s->prefault && std::find(bounce_out.begin(), bounce_out.end(), 1) != bounce_out.end()) {
        for (const auto& piece : pieces) {
            for (const Member& m : piece) {
                if (!bounce_out[m.tensor]) continue;
                const gq_tensor_t& t = tensors[m.tensor];
                const TypeInfo& ti = info[m.tensor];
                const size_t nvals = static_cast<size_t>(m.units) * ti.unit_values;
                if (ti.block_values == 0) {
                    s->prefault->submit(static_cast<uint8_t*>(static_cast<void*>(t.values)) + m.unit0 * ti.unit_bytes,
                                        nvals * ti.unit_bytes);
                    continue;
                }
                if (out_mask & GQ_OUT_CODES) s->prefault->submit(static_cast<uint8_t*>(t.codes) + m.unit0 * ti.unit_values, nvals);
                if (out_mask & GQ_OUT_F32) s->prefault->submit(t.values + m.unit0 * ti.unit_values, 4 * nvals);
            }
        }
    }

    struct Copy {
        void* dst;
        const void* src;
        size_t bytes;
    };
    std::vector<std::pair<gq::GqDesc, int>> items;
    std::vector<CopyJob> fill;
    std::vector<Copy> h2d, d2h;
    std::vector<CopyJob> drain[kSlots];
    auto drain_piece = [&](size_t p) -> int {
        std::vector<CopyJob>& jobs = drain[p % kSlots];
        if (jobs.empty()) return GQ_OK;
        const int e = cuda_status(cudaEventSynchronize(s->done[p % kSlots]));
        if (e != GQ_OK) return e;
        s->pool->run(jobs);
        jobs.clear();
        return GQ_OK;
    };
    for (size_t p = 0; p < pieces.size(); ++p) {
        const int k = static_cast<int>(p % kSlots);
        cudaStream_t stream = s->stream[k];
        uint8_t* base = s->slot[k];
        uint8_t* pin = s->pinned[k];
        size_t off = 0;
        items.clear();
        fill.clear();
        h2d.clear();
        d2h.clear();
        // an output region at slot offset `o`: straight to the caller's pinned buffer, or
        // through the pinned slot and a host copy afterwards
        auto out_region = [&](bool bounce, void* host, size_t o, size_t bytes) {
            if (bounce) {
                d2h.push_back({pin + o, base + o, bytes});
                drain[k].push_back({host, pin + o, bytes});
            } else {
                d2h.push_back({host, base + o, bytes});
            }
        };
        for (const Member& m : pieces[p]) {
            const gq_tensor_t& t = tensors[m.tensor];
            const TypeInfo& ti = info[m.tensor];
            const size_t src_bytes = static_cast<size_t>(m.units) * ti.unit_bytes;
            const uint8_t* hsrc = static_cast<const uint8_t*>(t.src) + m.unit0 * ti.unit_bytes;
            uint8_t* dsrc = base + off;
            if (bounce_in[m.tensor]) {
                fill.push_back({pin + off, hsrc, src_bytes});
                h2d.push_back({dsrc, pin + off, src_bytes});
            } else {
                h2d.push_back({dsrc, hsrc, src_bytes});
            }
            off = round_up(off + src_bytes);
            const bool bo = bounce_out[m.tensor];
            gq_tensor_t dt = t;
            dt.rows = m.units * ti.unit_values / t.cols;   // whole rows for a permuted tensor
            if (t.perm_heads > 0) dt.perm_heads = static_cast<int32_t>(dt.rows / (t.rows / t.perm_heads));
            dt.src = dsrc;
            dt.src_bytes = src_bytes;
            dt.diag = host_diags ? s->d_diag + m.tensor : nullptr;
            const int64_t nvals = m.units * ti.unit_values;
            if (ti.block_values == 0) {
                const size_t vb = static_cast<size_t>(nvals) * ti.unit_bytes;
                dt.values = reinterpret_cast<float*>(base + off);
                out_region(bo, static_cast<uint8_t*>(static_cast<void*>(t.values)) + m.unit0 * ti.unit_bytes, off, vb);
                off = round_up(off + vb);
            } else {
                if (out_mask & GQ_OUT_CODES) {
                    dt.codes = base + off;
                    out_region(bo, static_cast<uint8_t*>(t.codes) + m.unit0 * ti.unit_values, off,
                               static_cast<size_t>(nvals));
                    off = round_up(off + nvals);
                    dt.scales = reinterpret_cast<float*>(base + off);
                    const int64_t nsc = nvals / ti.block_values;
                    out_region(bo, t.scales + m.unit0 * (ti.unit_values / ti.block_values), off,
                               static_cast<size_t>(4 * nsc));
                    off = round_up(off + 4 * nsc);
                }
                if (out_mask & GQ_OUT_F32) {
                    dt.values = reinterpret_cast<float*>(base + off);
                    out_region(bo, t.values + m.unit0 * ti.unit_values, off, static_cast<size_t>(4 * nvals));
                    off = round_up(off + 4 * static_cast<size_t>(nvals));
                }
            }
            // rows of a piece: whole rows are not required (rows only matter for the
            // permutation, whose pieces are whole heads); present the piece as one row
            if (t.perm_heads == 0) {
                dt.rows = 1;
                dt.cols = nvals;
            }
            items.emplace_back(make_desc(dt, ti, m.units), t.type);
        }
        // host side of the input first (once the slot's previous piece, which may still be
        // reading the pinned slot, has finished), then the piece's GPU work on its stream
        if (!fill.empty()) {
            if (p >= kSlots && (st = cuda_status(cudaEventSynchronize(s->done[k]))) != GQ_OK) return fail(st);
            s->pool->run(fill);
        }
        for (const Copy& c : h2d) {
            st = cuda_status(cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyHostToDevice, stream));
            if (st != GQ_OK) return fail(st);
        }
        st = launch_grouped(items, out_mask, stream);
        if (st != GQ_OK) return fail(st);
        for (const Copy& c : d2h) {
            st = cuda_status(cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyDeviceToHost, stream));
            if (st != GQ_OK) return fail(st);
        }
        if ((st = cuda_status(cudaEventRecord(s->done[k], stream))) != GQ_OK) return fail(st);
        // while this piece runs, hand the previous piece's results to the caller
        if (p >= 1 && (st = drain_piece(p - 1)) != GQ_OK) return fail(st);
    }
    if (!pieces.empty() && (st = drain_piece(pieces.size() - 1)) != GQ_OK) return fail(st);
    for (int k = 0; k < kSlots; ++k) {
        st = cuda_status(cudaStreamSynchronize(s->stream[k]));
        if (st != GQ_OK) return fail(st);
    }
    if (s->prefault) s->prefault->cancel();
    if ((st = kernels_ok()) != GQ_OK) return st;
    if (host_diags != nullptr && count > 0) {
        // every stream's kernels have finished: read the maxima
        st = cuda_status(cudaMemcpy(host_diags, s->d_diag, sizeof(gq_diag_t) * count, cudaMemcpyDeviceToHost));
        if (st != GQ_OK) return st;
    }
    return GQ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Allocation-free host-buffer conversion
//
// Some callers cannot allocate device memory at the point where they convert weights: a
// process whose device memory is already handed out to another allocator (a framework's
// caching pool, a fixed budget shared with a runtime) must not call cudaMalloc, because it
// can fail there or implicitly synchronize the whole device.  For them this entry point
// stages everything in one fixed device array that is part of the library image: no
// cudaMalloc, cudaFree, stream or event creation, and no host heap allocation.
// ---------------------------------------------------------------------------------------

// The staging array.  Every GPU that loads the library holds these bytes until the
// process exits.  The first kNoAllocDiagBytes hold the per-tensor diagnostics.
constexpr size_t kNoAllocBytes = GQ_NOALLOC_SCRATCH_BYTES;
constexpr size_t kNoAllocDiagBytes = size_t(64) << 10;
static __device__ __align__(256) uint8_t gq_noalloc_scratch[kNoAllocBytes];

namespace {

// Per-device state: the array's device address (set up once, with the device current)
// and the batch parameter block, both in static storage.  The mutex serializes calls of
// this process on one device; all of them share the array.
struct NoAllocDevice {
    std::mutex mu;
    uint8_t* scratch = nullptr;
    gq::GqBatch batch;
};
NoAllocDevice g_noalloc[64];

int noalloc_setup(int device, NoAllocDevice** out) {
    if (device < 0 || device >= 64) return GQ_ERR_ARG;
    NoAllocDevice& nd = g_noalloc[device];
    if (nd.scratch == nullptr) {
        // In host code the symbol is only a stand-in: its device address must be asked
        // for, once per device, while that device is current.
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, gq_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr) return cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
        nd.scratch = static_cast<uint8_t*>(ptr);
    }
    *out = &nd;
    return GQ_OK;
}

}  // namespace

extern "C" {

int gq_convert_host_noalloc(int32_t device, const gq_tensor_t* tensors, int32_t count, int32_t out_mask,
                            gq_diag_t* host_diags, void* stream) {
    if (count < 0) return GQ_ERR_ARG;
    if (count > 0 && tensors == nullptr) return GQ_ERR_NULL;
    if (!valid_mask(out_mask)) return GQ_ERR_ARG;
    if (host_diags != nullptr && static_cast<size_t>(count) * sizeof(gq_diag_t) > kNoAllocDiagBytes)
        return GQ_ERR_SIZE;   // more tensors than the diagnostics area holds
    if (device < 0 || device >= 64) return GQ_ERR_ARG;
    const size_t staging = kNoAllocBytes - kNoAllocDiagBytes;
    // validate everything before any device work
    for (int i = 0; i < count; ++i) {
        const gq_tensor_t& t = tensors[i];
        TypeInfo ti;
        int64_t nv = 0, nu = 0;
        const int st = shape_check(t, &ti, &nv, &nu);
        if (st != GQ_OK) return st;
        if (nv == 0) continue;
        if (t.src == nullptr) return GQ_ERR_NULL;
        if (ti.block_values == 0) {
            if (t.values == nullptr) return GQ_ERR_NULL;
        } else {
            if ((out_mask & GQ_OUT_CODES) && (t.codes == nullptr || t.scales == nullptr)) return GQ_ERR_NULL;
            if ((out_mask & GQ_OUT_F32) && t.values == nullptr) return GQ_ERR_NULL;
        }
        // the smallest piece (one unit, or one head of a permuted tensor) must fit
        const size_t fp = unit_footprint(ti, out_mask);
        const int64_t upr = t.cols / ti.unit_values;
        const int64_t min_units = t.perm_heads > 0 ? (t.rows / t.perm_heads) * upr : 1;
        if (static_cast<size_t>(min_units) * fp + 4 * kAlign > staging) return GQ_ERR_SIZE;
    }
    // the lock is taken before the device scope, so the caller's device is restored first
    // and the mutex is released last, after any queued work has drained
    std::lock_guard<std::mutex> lock(g_noalloc[device].mu);
    const DeviceScope scope(device);
    int st = scope.status();
    if (st != GQ_OK) return st;
    NoAllocDevice* nd = nullptr;
    if ((st = noalloc_setup(device, &nd)) != GQ_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    gq_diag_t* d_diag = reinterpret_cast<gq_diag_t*>(nd->scratch);
    uint8_t* base = nd->scratch + kNoAllocDiagBytes;
    // Once anything is queued, an error return first waits for the stream (its status is
    // not what the caller needs: the first error is), so that no copy still lands in the
    // caller's buffers and no queued work still uses the array after the call returns.
    bool queued = false;
    auto fail = [&](int e) {
        if (queued) {
            cudaStreamSynchronize(s);
            cudaGetLastError();
        }
        return e;
    };
    if (host_diags != nullptr && count > 0) {
        // the array keeps the previous call's contents: the maxima must start at zero
        st = cuda_status(cudaMemsetAsync(d_diag, 0, sizeof(gq_diag_t) * count, s));
        if (st != GQ_OK) return fail(st);
        queued = true;
    }
    gq::GqBatch& b = nd->batch;
    for (int i = 0; i < count; ++i) {
        const gq_tensor_t& t = tensors[i];
        TypeInfo ti;
        int64_t nv = 0, units = 0;
        shape_check(t, &ti, &nv, &units);
        if (nv == 0) continue;
        const size_t fp = unit_footprint(ti, out_mask);
        const int64_t upr = t.cols / ti.unit_values;
        // a permuted tensor is cut into whole heads, which the permutation keeps apart
        const int64_t step = t.perm_heads > 0 ? (t.rows / t.perm_heads) * upr : 1;
        int64_t per_piece = static_cast<int64_t>((staging - 4 * kAlign) / fp);
        per_piece = (per_piece / step) * step;
        for (int64_t u0 = 0; u0 < units; u0 += per_piece) {
            const int64_t n = std::min<int64_t>(per_piece, units - u0);
            const int64_t nvals = n * ti.unit_values;
            size_t off = 0;
            gq_tensor_t dt = t;
            dt.src = base;
            dt.src_bytes = static_cast<size_t>(n) * ti.unit_bytes;
            off = round_up(off + dt.src_bytes);
            if (t.perm_heads > 0) {
                dt.rows = n / upr;
                dt.perm_heads = static_cast<int32_t>(dt.rows / (t.rows / t.perm_heads));
            } else {
                dt.rows = 1;
                dt.cols = nvals;
            }
            dt.diag = host_diags ? d_diag + i : nullptr;
            st = cuda_status(cudaMemcpyAsync(base, static_cast<const uint8_t*>(t.src) + u0 * ti.unit_bytes,
                                             dt.src_bytes, cudaMemcpyHostToDevice, s));
            if (st != GQ_OK) return fail(st);
            queued = true;
            void* h_dst[3] = {nullptr, nullptr, nullptr};
            const void* d_src[3] = {nullptr, nullptr, nullptr};
            size_t n_bytes[3] = {0, 0, 0};
            if (ti.block_values == 0) {
                dt.values = reinterpret_cast<float*>(base + off);
                n_bytes[0] = static_cast<size_t>(nvals) * ti.unit_bytes;
                h_dst[0] = reinterpret_cast<uint8_t*>(t.values) + u0 * ti.unit_bytes;
                d_src[0] = dt.values;
            } else {
                if (out_mask & GQ_OUT_CODES) {
                    dt.codes = base + off;
                    off = round_up(off + nvals);
                    dt.scales = reinterpret_cast<float*>(base + off);
                    const int64_t nsc = nvals / ti.block_values;
                    off = round_up(off + 4 * nsc);
                    h_dst[0] = static_cast<uint8_t*>(t.codes) + u0 * ti.unit_values;
                    d_src[0] = dt.codes;
                    n_bytes[0] = static_cast<size_t>(nvals);
                    h_dst[1] = t.scales + u0 * (ti.unit_values / ti.block_values);
                    d_src[1] = dt.scales;
                    n_bytes[1] = static_cast<size_t>(4 * nsc);
                }
                if (out_mask & GQ_OUT_F32) {
                    dt.values = reinterpret_cast<float*>(base + off);
                    h_dst[2] = t.values + u0 * ti.unit_values;
                    d_src[2] = dt.values;
                    n_bytes[2] = static_cast<size_t>(4 * nvals);
                }
            }
            b.n = 1;
            b.total_tiles = gq::tiles_for(t.type, n);
            b.d[0] = make_desc(dt, ti, n);
            b.d[0].tile_begin = 0;
            const int e = gq::launch_batch(t.type, out_mask, b, s);
            if (e != 0) return fail(cuda_status(e));
            for (int k = 0; k < 3; ++k) {
                if (n_bytes[k] == 0) continue;
                st = cuda_status(cudaMemcpyAsync(h_dst[k], d_src[k], n_bytes[k], cudaMemcpyDeviceToHost, s));
                if (st != GQ_OK) return fail(st);
            }
            // the next piece overwrites the staging bytes: stream order puts its copy
            // after these reads
        }
    }
    if (host_diags != nullptr && count > 0) {
        st = cuda_status(cudaMemcpyAsync(host_diags, d_diag, sizeof(gq_diag_t) * count, cudaMemcpyDeviceToHost, s));
        if (st != GQ_OK) return fail(st);
    }
    if ((st = cuda_status(cudaStreamSynchronize(s))) != GQ_OK) return st;
    return kernels_ok();
}

}  // extern "C"
