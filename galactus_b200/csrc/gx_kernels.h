// Host-side declarations of the kernel launchers (internal to the library).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "gx_formats.h"

namespace gx {

constexpr int kRowsThreads = 128;
constexpr uint32_t kMaxSmem = 227 * 1024;
constexpr int kInlineIds = 64;
constexpr int kDecodeMaxThreads = 256;

// Parameters of the row-tile kernel (all three modes). Byte offsets of the
// shared-memory regions are filled by rows_smem_layout().
struct RowsParams {
    const uint8_t * w0;      // weights of the (first) role, expert e at w0 + e*nb02
    const uint8_t * w1;      // up weights (GATE_UP)
    int64_t nb01, nb02;
    int32_t ne00, ne01, n_as;
    const float * src;       // f32 activations, row (t, i) at src + t*nb12 + i*nb11
    int64_t nb11, nb12;
    int32_t ne11;
    const int32_t * ids;     // i32 [k, T], token stride nbi1 bytes (device), unless use_inline
    int64_t nbi1;
    int32_t k, T;
    int32_t use_inline;
    int32_t inline_ids[kInlineIds];
    const float * rw;        // router weights [k, T] (DOWN_COMBINE)
    float * dst;
    int32_t R;               // rows per expert tile
    int32_t act;             // GX_ACT_*
    float alpha, limit;
    int32_t act_pitch, n_act;
    uint32_t bar_off, tile_off, act_off, terms_off, dots_off;
};

enum { kModePlain = 0, kModeGateUp = 1, kModeDownCombine = 2 };

// ------------------------------------------------------------ split layout

struct ActLayout {
    int32_t d_off;    // byte offset of the scales (fp16 for Q8_0, f32 for Q8_K)
    int32_t bs_off;   // byte offset of the Q8_K block sums (int16 per 16 elements)
    int32_t pitch;    // bytes per row, multiple of 16
};

GX_HD int32_t align16i(int64_t v) { return (int32_t)((v + 15) / 16 * 16); }

GX_HD ActLayout act_layout(int vdt, int n) {
    ActLayout a;
    a.d_off = n;
    if (vdt == GX_T_Q8_0) {
        a.bs_off = n + (n / 32) * 2;
        a.pitch = align16i(a.bs_off);
    } else {
        a.bs_off = n + (n / 256) * 4;
        a.pitch = align16i(a.bs_off + (n / 16) * 2);
    }
    return a;
}

struct DecodeParams {
    const uint8_t * w0;        // gate (GATE_UP) or down (DOWN) role base of slot 0
    const uint8_t * w1;        // up role base (GATE_UP)
    int64_t nb01, nb02;        // row bytes, record stride
    int32_t ne00, ne01;        // input length, output rows per expert
    int32_t n_as;              // slots of the layer
    int32_t k, T;
    int32_t R;                 // rows per expert per stage
    int32_t S;                 // pipeline stages
    int32_t row_copy;          // 1: one bulk copy per row (pitch_w), 0: one per R-row tile
    int32_t pitch_w;           // shared-memory bytes between rows of a stage
    int32_t stage_bytes;
    int32_t n_units;
    const int32_t * ids;       // slot ids [T, k] (device) unless use_inline
    int32_t use_inline;
    int32_t inline_ids[kInlineIds];
    const uint8_t * aq;        // quantized input rows (split layout)
    ActLayout al;              // layout of aq rows
    int32_t a_rows;            // aq rows loaded per token (1 for GATE_UP, k for DOWN)
    // GATE_UP outputs
    float * act_f32;           // [T*k, ne01]
    uint8_t * act_q;           // [T*k, al2.pitch] split-layout quantized activations for the down projection
    ActLayout al2;
    int32_t vdt2, qblk;        // down input quant type and its block rows
    int32_t * counters;        // [T*k, ne01/qblk], zero between calls
    int32_t act;
    float alpha, limit;
    // DOWN outputs
    const float * rw;          // router weights [T, k]
    float * out;               // [T, ne01]
    uint32_t act_off, stage_off, dots_off, flag_off;
};

// ------------------------------------------------------------ stack kernel

// One layer of a persistent stack launch (device-resident table).
struct StackLayer {
    const uint8_t * wg;        // gate role base of slot 0
    const uint8_t * wu;        // up role base of slot 0
    const uint8_t * wd;        // down role base of slot 0
    const float * x;           // [T, H] input rows
    const float * rw;          // [T, k] router weights
    float * out;               // [T, H]
    const int32_t * slots;     // [T, k] slot ids
    uint8_t * xq;              // T split-layout rows of x (alx.pitch)
    float * act;               // [T*k, I] activation (f32)
    uint8_t * actq;            // T*k split-layout rows of act (ald.pitch)
    int32_t * cnt;             // [T*k, I/qblk] gate/up units finished per Q8 block
    int64_t nb02;              // record stride (bytes between slots)
    int32_t n_as;              // slots of the layer
    int32_t pad;
};

constexpr int kStackMaxConsumers = 16;  // ring stages
constexpr int kStackMaxWarps = 16;      // consumer warps (any row mode)
// consumer warps of a row mode: the MXFP4 rows (mode 3) run four warps per
// 32-row job, the others at most twelve (their register budgets)
GX_HD constexpr int stack_max_warps(int row_mode) { return row_mode == 3 ? 16 : 12; }
constexpr int kStackProducers = 2;      // weight producer warps (even and odd jobs)
constexpr int kStackMaxLayers = 128;   // the layer table travels in the kernel parameters
constexpr int kStackBufs = 2;          // activation buffers per kind (gate/up inputs, down inputs)

struct StackParams {
    int32_t * q_done;          // [NL]   1 once x_L is quantized (row mode 5: its blocks quantized, T*H/32 when done)
    int32_t * gu_done;         // [NL*T] quantized down-input blocks per token (k*I/qblk when complete)
    int32_t NL, k, T, H, I;
    int64_t nb01_g, nb01_d;    // gate/up and down row bytes
    int32_t Rg;                // gate (and up) rows per gate/up job
    int32_t Rd;                // output rows per down job (k*Rd = 32 weight rows, or 16 in row mode 2)
    int32_t C;                 // ring stages
    int32_t W;                 // consumer warps (may exceed C)
    int32_t skew;              // down jobs of layer L follow the gate/up jobs of layer L+skew
    int32_t row_copy_d, pitch_d;
    int32_t row_mode;          // 0: two-lane Q8_0 rows, 1: octet rows, 2: two-lane Q4_K/Q6_K rows, 3: MXFP4 rows on
                               // the CUDA cores, 4: MXFP4 rows on the tensor cores (activations as e4m3 digit rows)
    int32_t gu_copies;         // 4 (modes 0, 2): gate/up job in 4 tiles of 4 rows (gate 0-3, 4-7, up 0-3,
                               //    4-7) at gu_tile[0..3], staggered so quarter-warp loads hit distinct
                               //    bank groups; 2 (mode 1): gate rows 0-7 at gu_tile[0], up rows at gu_tile[1]
    int32_t gu_tile[4];
    int32_t stage_bytes;       // weight rows of one job
    ActLayout alx, ald;        // layouts of xq rows and actq rows
    int32_t qblk;              // elements per Q8 block of the down input
    int32_t n_gu, n_d;         // gate/up and down jobs per layer
    int32_t act;
    float alpha, limit;
    uint32_t bar_off, meta_off, stage_off, xbuf_off, dbuf_off, wt_off, slots_off, dots_off;
    int32_t need_grid;         // 1: IQ1_S rows, the 16 KB codebook copied to shared memory at grid_off
    int32_t split;             // warps per job: 4 for MXFP4 jobs, 2 for octet jobs and 32-row two-lane K-quant
                               // down jobs, else 1
    uint32_t grid_off;
    uint32_t tc_off;           // row modes 4, 5: their shared-memory region
    int32_t nbuf_d;            // down-input buffers (kStackBufs, or 1 in row mode 4)
    int32_t tc_na;             // row mode 4: A-tile slots (MMA steps in flight); row mode 5: ring stages
    const CUtensorMap * t5_maps;   // row mode 5: [NL][3] codes of gate (64-row boxes), up (64), down (32)
    uint32_t t5_jobs_off;      // row mode 5: the CTA's job table in shared memory (8 bytes per job)
    int32_t t5_jobs;           // its capacity (jobs past it are computed where used)
    StackLayer layers[kStackMaxLayers];
};

// Expert-grouped prefill kernels (gx_prefill.cuh).
struct PrefillParams {
    const uint8_t * w0;        // gate (MODE 0) or down (MODE 1) role base of slot 0
    const uint8_t * w1;        // up role base (MODE 0)
    int64_t nb01, nb02;        // row bytes, record stride
    int32_t K;                 // row length in elements (multiple of 256)
    int32_t n_as;              // slots of the layer
    int32_t tile[4];           // staggered offsets of the four 4-row weight tiles
    uint32_t act_off;          // shared-memory offset of the two activation chunks
    int32_t n_units;
    const int32_t * unit_slot; // [n_units]
    const int32_t * unit_row0; // [n_units] first weight row of the unit (MODE 0: of 8 gate/up rows)
    const int32_t * seg_start; // [n_as+1] the slot's range in the sorted pair arrays
    const int32_t * pair_src;  // [P] activation row of each sorted pair (MODE 0: token, MODE 1: pair)
    const int32_t * pair_dst;  // [P] output row (the pair index t*k+s)
    const uint8_t * aq;        // activation rows, split layout
    ActLayout al;
    float * out;               // MODE 0: act [P, I]; MODE 1: y [P, H]
    int64_t out_ld;
    int32_t act;
    float alpha, limit;
};

uint32_t prefill_layout(PrefillParams & p);
cudaError_t launch_prefill(int mode, const PrefillParams & p, uint32_t smem, cudaStream_t stream);

// Tensor-core prefill (gx_mma.cuh): pair chunks of <= 16 pairs of one expert.
constexpr int kMmaRows = 128;          // weight rows per unit (MMA M)
constexpr int kMmaTok = 16;            // (token, slot) pairs per chunk
constexpr int kMmaN = 4 * kMmaTok;     // MMA N: four lane copies per pair
constexpr int kMmaMaxBlocks = 64;      // Q8_0 blocks per row at most (K <= 2048)
struct MmaPrepParams {
    const int32_t * chunk_first;   // [chunks] first sorted-pair index
    const int32_t * chunk_count;   // [chunks] pairs in the chunk (<= 16)
    const int32_t * pair_src;      // [P] activation row of each sorted pair
    const uint8_t * aq;            // activation rows (Q8_0 split layout)
    ActLayout al;
    int32_t nblk;                  // Q8_0 blocks per activation row
    uint8_t * btiles;              // [chunks][nblk][64 x 32] masked B tiles
    float * dyt;                   // [chunks][nblk][16] block scales
};
struct MmaParams {
    // weight rows of every slot as a 3-D tensor of 16-bit words: x = word in
    // the row (nb01 / 2), y = row (MODE 0: the I gate rows then the I up rows,
    // contiguous in the record; MODE 1: the H down rows), z = slot; boxes of
    // 136 words (8 Q8_0 blocks) x 64 (MODE 0) or 128 (MODE 1) rows
    CUtensorMap tmap;
    int32_t up_row0;               // MODE 0: row of up row 0 in the tensor (I)
    int64_t nb01;                  // row bytes
    int32_t nblk;                  // Q8_0 blocks per weight row (a multiple of 8, at most 64)
    int32_t n_rt;                  // row tiles per chunk (units = chunks * n_rt)
    const int32_t * chunk_slot;    // [chunks]
    const int32_t * chunk_first;   // [chunks]
    const int32_t * chunk_count;   // [chunks]
    const int32_t * pair_dst;      // [P] output row of each sorted pair
    const uint8_t * btiles;
    const float * dyt;
    float * out;                   // MODE 0: act [P, I]; MODE 1: y [P, H]
    int64_t out_ld;
    int32_t act;
    float alpha, limit;
};
cudaError_t launch_mma_bprep(const MmaPrepParams & p, int n_chunks, cudaStream_t stream);
cudaError_t launch_prefill_mma(int mode, const MmaParams & p, int n_units, cudaStream_t stream);
// the tensor-core prefill's constraints: Q8_0 weights and activations, K a multiple of 256 (8 blocks) up to 2048
bool prefill_mma_supported(int type_gate, int type_down, int64_t H, int64_t I);

uint32_t stack_layout(StackParams & p, int & threads);
bool stack_types_supported(int type_gate, int type_down);
// Resident CTAs per SM of the stack kernel for this layout (0 on error).
cudaError_t prepare_stack(int type_gate, int type_down, const StackParams & p, int threads, uint32_t smem, int & per_sm);
cudaError_t launch_stack(int type_gate, int type_down, const StackParams & p, int grid, int threads, uint32_t smem,
                         cudaStream_t stream);
int device_sms();

uint32_t decode_layout(int mode, DecodeParams & p, int & threads);
cudaError_t launch_decode(int type, int mode, DecodeParams & p, cudaStream_t stream, bool pdl);
cudaError_t prepare_decode(int type, int mode, DecodeParams p);
cudaError_t launch_quant_split(int vdt, const float * src, int ne0, int64_t nrows, int64_t nb1, uint8_t * dst,
                               cudaStream_t stream, bool pdl);

uint32_t rows_smem_layout(int type, int mode, RowsParams & p);
cudaError_t launch_rows(int type, int mode, RowsParams & p, dim3 grid, cudaStream_t stream);
cudaError_t launch_quantize_rows(int vdt, const float * src, int ne0, int64_t nrows, int64_t nb1, uint8_t * dst,
                                 int64_t pitch, cudaStream_t stream);
cudaError_t launch_swiglu(const float * g, const float * u, float * out, int64_t n, cudaStream_t stream);
cudaError_t launch_swiglu_oai(const float * g, const float * u, float * out, int64_t n, float alpha, float limit,
                              cudaStream_t stream);
cudaError_t launch_expf(const float * x, float * y, int64_t n, cudaStream_t stream);
cudaError_t launch_combine(const float * y, const float * w, float * out, int64_t H, int k, int64_t T, cudaStream_t stream);
cudaError_t launch_move_rows(const float * src, const int32_t * idx, int64_t n, int64_t H, float * dst, bool scatter,
                             cudaStream_t stream);
cudaError_t launch_fill(float * dst, int64_t n, float v, cudaStream_t stream);
// dst[j] = row rows[j] of the [*, H] matrix at ptrs[layers[j]] (gather over a pointer table)
cudaError_t launch_gather_ptrs(const float * const * ptrs, const int32_t * layers, const int32_t * rows, int64_t n,
                               int64_t H, float * dst, cudaStream_t stream);
// Row mode 5 (TMA-fed tensor-core MXFP4 stack jobs): MMA issuer warps (1,
// 10, 11, then 14, ...) and the CTA's warps (2 chunk producers, a scale
// producer, 2 input producers, 4 epilogue and 2 tail warps besides the issuers)
constexpr int kT5Issuers = 4;
constexpr int kT5Warps = 11 + kT5Issuers;

// One record's MXFP4 matrices (down, gate, up) for the tensor-core layout:
// per matrix the codes in TMA-box order [tile of trows rows][chunk of 4
// blocks][row of the tile][64 bytes: the 16 code bytes of each of the 4
// blocks] (each box one contiguous run; rows padded to whole chunks), then
// the block scales [rows][nb].
struct Mxfp4TcMats {
    int64_t off[3];    // matrix offsets in the source (GGUF) record
    int64_t doff[3];   // matrix offsets in the tensor-core record
    int32_t rows[3];
    int32_t nb[3];     // 32-element blocks per row
    int32_t trows[3];  // rows per tile (TMA box rows)
};
// code bytes per row of nb blocks in the tensor-core layout (whole chunks)
GX_HD constexpr int32_t mxfp4_tc_cstride(int32_t nb) { return ((nb + 3) / 4) * 64; }
cudaError_t launch_mxfp4_tc_layout(const uint8_t * src, uint8_t * dst, const Mxfp4TcMats & m, cudaStream_t stream);
// out[i] = out[i] + b[i] (one rounding per element)
cudaError_t launch_add_inplace(float * out, const float * b, int64_t n, cudaStream_t stream);
// router: logits [rows, ld] -> ids/w [rows, k] (+ slots through table); rows = n_layers * T
constexpr int kRouterWarps = 4;
constexpr int kRouterMaxExperts = 1024;
constexpr int kRouterMaxUsed = 32;
constexpr int kRouterMaxGroups = 32;
struct RouterLaunch {
    const float * logits;
    int64_t ld;
    const float * bias;
    const int32_t * table;
    int32_t * ids;
    float * w;
    int32_t * slots;
    int64_t T, n_layers;
    int E, k, gating, groups, group_used, norm, scale_on;
    float scale;
};
cudaError_t launch_router(const RouterLaunch & r, cudaStream_t stream);
cudaError_t launch_synth_normal(float * dst, int64_t n, uint64_t seed, uint64_t stream_id, float sigma, cudaStream_t stream);
cudaError_t launch_synth_weights(int type, void * dst, int64_t ne00, int64_t n_rows, uint64_t seed, uint64_t stream_id,
                                 float sigma, cudaStream_t stream);
cudaError_t read_and_clear_device_error(int * code);
uint64_t synth_key(uint64_t seed, uint64_t stream_id);

}  // namespace gx
