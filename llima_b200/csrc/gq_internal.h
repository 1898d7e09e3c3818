// Internal types shared by the kernels and the C ABI layer.
#pragma once

#include <stdint.h>

#include "../../include/gguf_b200.h"

namespace gq {

// One tensor of a batch launch as the kernels see it.  Work is cut into tiles of a
// fixed number of stored units; tiles are numbered across the batch and tile_begin is
// this tensor's first tile.
struct GqDesc {
    const uint8_t* src;
    uint8_t* codes;
    float* scales;
    float* values;
    gq_diag_t* diag;
    int64_t n_units;
    int64_t tile_begin;
    int64_t units_per_row;   // for the head permutation
    int32_t perm_heads;      // 0: no permutation
    int32_t rows_per_head;   // head_dim of the permuted rows
    // 32-bit division by units_per_row and rows_per_head as multiply-high and shifts
    // (Granlund and Montgomery, "Division by invariant integers using multiplication",
    // 1994, figure 4.1); upr_mul == 0 when the unit indices do not fit (64-bit path)
    uint32_t upr_mul, upr_shift;   // shift: sh1 | sh2 << 8
    uint32_t rph_mul, rph_shift;
};

// Multiplier and shifts of the invariant-divisor method for 32-bit n and divisor d >= 1:
// l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1, sh1 = min(l, 1), sh2 = max(l - 1, 0).
inline void fast_div_params(uint32_t d, uint32_t& mul, uint32_t& shift) {
    int l = 0;
    while (l < 32 && (uint64_t(1) << l) < d) ++l;
    mul = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
    shift = static_cast<uint32_t>(l < 1 ? l : 1) | (static_cast<uint32_t>(l > 1 ? l - 1 : 0) << 8);
}

// Kernel parameter block (passed by value; larger than 4 KB needs CUDA >= 12.1).
constexpr int kMaxDesc = 256;

struct GqBatch {
    int32_t n;
    int32_t pad;
    int64_t total_tiles;
    GqDesc d[kMaxDesc];
};

// kOutSmem (internal): the codes and scales go to a shared-memory tile instead of the
// tensor's global buffers (the fused Modalix layout writer transposes them from there)
enum : int { kOutCodes = GQ_OUT_CODES, kOutF32 = GQ_OUT_F32, kOutSmem = 4 };

// One tensor converted straight into the Modalix weight layout (gq_convert_modalix).
struct GqModalix {
    const uint8_t* src;       // GGUF bytes, rows x units_per_row stored units
    uint8_t* out_codes;       // (cols, rows_padded)
    float* out_scales;        // (cols / block, rows_padded)
    gq_diag_t* diag;          // optional requantization diagnostics
    int64_t rows, cols, rows_padded;
    int64_t units_per_row;
    uint32_t n_col_tiles, n_tiles;
    uint32_t ncol_mul, ncol_shift;   // division by n_col_tiles (fast_div_params)
    int32_t head_dim;         // > 0: llama q/k head permutation with heads of this size
    uint32_t tile_begin;      // first tile of this tensor in its batch
};

// Tensors of one GGML type converted into the Modalix layout by one launch.
constexpr int kMaxModalix = 128;
struct GqModalixBatch {
    int32_t n;
    uint32_t total_tiles;
    GqModalix d[kMaxModalix];
};

// launch entry points implemented in gq_kernels.cu
// sticky kernel error flags of the current device (read, then cleared when `clear`)
int kernel_errors(bool clear, uint32_t* flags);
int launch_batch(int type, int out_mask, const GqBatch& batch, void* stream);
int64_t tiles_for(int type, int64_t n_units);
int launch_modalix(int type, const GqModalixBatch& b, void* stream);
constexpr int kModalixRows = 64;    // output channels per tile of the fused layout writer
constexpr int kModalixCols = 256;   // input channels per tile
int launch_layout(const uint8_t* codes, const float* scales, int64_t rows, int64_t cols, int64_t nb,
                  int64_t rows_padded, uint8_t* out_codes, float* out_scales, void* stream);
int64_t embed_max_row_bytes();
int launch_embed(int type, bool from_f32, const uint8_t* src, int64_t rows, int64_t cols, int64_t row_bytes,
                 float embed_scale, int quantize, int8_t* codes, uint16_t* scales, float* values, int64_t src_bytes,
                 void* stream);
int launch_requant(const float* bc, const int8_t* codes, int64_t n_blocks, int block, int bits,
                   float* out_scales, int8_t* out_codes, gq_diag_t* diag, void* stream);
// implemented in gq_fields.cu
int launch_fields(int type, const uint8_t* src, int64_t n_units, float* sup, int8_t* blk, int8_t* vals,
                  void* stream);
int launch_superblocks(const float* sup, const void* blk, int blk_bytes, int64_t n_super, int nb, int k,
                       uint16_t* out_f16, float* out_f32, void* stream);

}  // namespace gq
