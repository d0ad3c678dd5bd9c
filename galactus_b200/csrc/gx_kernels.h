// Host-side declarations of the kernel launchers (internal to the library).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace gx {

constexpr int kRowsThreads = 128;
constexpr uint32_t kMaxSmem = 227 * 1024;
constexpr int kInlineIds = 64;

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

uint32_t rows_smem_layout(int type, int mode, RowsParams & p);
cudaError_t launch_rows(int type, int mode, RowsParams & p, dim3 grid, cudaStream_t stream);
cudaError_t launch_quantize_rows(int vdt, const float * src, int ne0, int64_t nrows, int64_t nb1, uint8_t * dst,
                                 int64_t pitch, cudaStream_t stream);
cudaError_t launch_swiglu(const float * g, const float * u, float * out, int64_t n, cudaStream_t stream);
cudaError_t launch_swiglu_oai(const float * g, const float * u, float * out, int64_t n, float alpha, float limit,
                              cudaStream_t stream);
cudaError_t launch_expf(const float * x, float * y, int64_t n, cudaStream_t stream);
cudaError_t launch_combine(const float * y, const float * w, float * out, int64_t H, int k, int64_t T, cudaStream_t stream);
cudaError_t launch_synth_normal(float * dst, int64_t n, uint64_t seed, uint64_t stream_id, float sigma, cudaStream_t stream);
cudaError_t launch_synth_weights(int type, void * dst, int64_t ne00, int64_t n_rows, uint64_t seed, uint64_t stream_id,
                                 float sigma, cudaStream_t stream);
cudaError_t read_and_clear_device_error(int * code);
uint64_t synth_key(uint64_t seed, uint64_t stream_id);

}  // namespace gx
