/*
 * galactus_b200 -- C-ABI of the B200 routed-expert FFN.
 *
 * This is the boundary a patched llama.cpp graph binds. Every entry point takes
 * plain pointers and sizes; device pointers are CUDA device addresses, streams
 * are cudaStream_t passed as void*. No entry point throws: each returns a
 * GX_* status code (0 = success).
 *
 * The op surface it replaces, in the reference's patched llama.cpp
 * (patches/galactus-h4-llamacpp.diff, cited by the diff's own line numbers):
 *   galactus_h4::init / create_exps / remap_ids      diff:2147-2150, 2260-2264, 2293-2296
 *   ggml_mul_mat_id on the expert tensors            diff:2161, 2170, 2179, 2188
 *   ggml_swiglu_split / GGML_GLU_OP_SWIGLU_OAI       diff:1461-1465
 * and, underneath the glue, the H4 engine:
 *   galactus::h4::ModelProfile                       src/h4/h4-profile.hpp:19-39
 *   galactus::h4::ExpertCache                        src/h4/h4-expert-cache.hpp:66-196
 *   galactus::h4::ExpertStore                        src/h4/h4-expert-store.hpp:27-117
 */
#ifndef GALACTUS_B200_H
#define GALACTUS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define GX_OK              0
#define GX_ERR_INVALID    -1  /* null pointer, bad size or stride */
#define GX_ERR_TYPE       -2  /* weight type without a bit-exact kernel (reference: decline, diff:53-96) */
#define GX_ERR_ALIGN      -3  /* ne00 not a multiple of 64 (Q8_0 family) or 256 (Q8_K family), or a
                                 tensor base/stride the kernels cannot stage (diff:181-187) */
#define GX_ERR_DOMAIN     -4  /* expert id outside [0, n_expert) */
#define GX_ERR_BATCH      -5  /* a micro-batch holds more distinct experts than the probation segment */
#define GX_ERR_SLOTS      -6  /* free list exhausted or a served key has no slot
                                 (src/h4/h4-expert-store.cpp:127-141; scripts/derive-remap-strides.py:70) */
#define GX_ERR_CUDA       -7  /* a CUDA runtime call failed */
#define GX_ERR_TIMEOUT    -8  /* a bounded device-side wait ran out */
#define GX_ERR_NOMEM      -9  /* device or pinned host allocation failed */
#define GX_ERR_COPY      -10  /* a host->HBM miss copy failed */
#define GX_ERR_STATE     -11  /* call out of order (e.g. no host tier) */
#define GX_ERR_DEVICE    -12  /* a kernel reported an error (see gx_device_error) */
#define GX_ERR_COMM      -13  /* an NCCL call failed or NCCL could not be loaded */

/* ggml type ids (ggml.h numbering) of the formats this library computes on */
#define GX_TYPE_Q8_0   8
#define GX_TYPE_Q4_K  12
#define GX_TYPE_Q6_K  14
#define GX_TYPE_Q8_K  15
#define GX_TYPE_IQ1_S 19
#define GX_TYPE_MXFP4 39

/* slot policies: GALACTUS_H4_CACHE_POLICY values (src/h4/h4-cache-plan.hpp:83-97) plus pure LRU */
#define GX_POLICY_AUTO      0  /* plan (when given) + frequency victim: the reference default */
#define GX_POLICY_UNIFORM   1  /* equal quota, SLRU with LRU victim (the shipped policy) */
#define GX_POLICY_PLAN      2  /* plan only, LRU victim */
#define GX_POLICY_FREQUENCY 3  /* equal quota, frequency victim */
#define GX_POLICY_LRU       4  /* one segment, least recently used victim (no reference counterpart) */

/* activations of the expert FFN */
#define GX_ACT_SWIGLU     0
#define GX_ACT_SWIGLU_OAI 1

const char * gx_status_string(int status);

/* Library build identity (kernel generation, target arch). */
const char * gx_version(void);

/* Select the CUDA device for the calling thread and load the device tables.
 * Returns GX_ERR_CUDA when no device is present. */
int gx_device_init(int device);

/* First error code recorded by a kernel on the current device since the last
 * call (0 if none), and clear it. Kernels record instead of trapping: an
 * out-of-domain expert id, or a bounded wait that ran out. */
int gx_device_error(int32_t * code_out);

/* ----------------------------------------------------------------- profile
 * MoE geometry of the routed layers (ModelProfile, src/h4/h4-profile.hpp:19-39).
 * record_bytes[i] is the 16 KiB-padded record of layer first_layer+i
 * (down | gate | up), record_bytes_raw[i] its useful bytes. */
typedef struct gx_profile {
    uint32_t first_layer;
    uint32_t last_layer;
    uint32_t experts;   /* experts per layer (<= 1024, the key encoding capacity) */
    uint32_t used;      /* experts selected per token */
    const uint64_t * record_bytes;
    const uint64_t * record_bytes_raw;
} gx_profile;

/* ------------------------------------------------------------ slot policy
 * The per-layer slot cache and slot ledger, host only: ExpertCache plus the
 * slot tables of ExpertStore (warm path, src/h4/h4-expert-store.cpp:197-211).
 * No device memory is touched; usable on any host. */
typedef struct gx_policy gx_policy;

typedef struct gx_serve_stats {
    uint32_t hits;
    uint32_t misses;
    uint32_t evictions;
    uint32_t distinct;
    uint64_t bytes_copied;   /* host->HBM bytes issued by this call */
} gx_serve_stats;

/* capacity_bytes: the whole cache budget; quota = capacity / sum of one record
 * per layer, capped at `experts` (src/h4/h4-expert-cache.cpp:68-135).
 * plan_quotas: optional per-layer quotas (NULL = uniform), validated against
 * the budget the uniform quota buys. */
int gx_policy_create(const gx_profile * profile, uint64_t capacity_bytes, double protected_fraction,
                     int policy, const uint32_t * plan_quotas, gx_policy ** out);
void gx_policy_destroy(gx_policy * policy);
int gx_policy_quota(const gx_policy * policy, uint32_t layer, uint32_t * quota,
                    uint32_t * protected_quota, uint32_t * probation_quota);
/* One micro-batch of one layer through the policy: begin_batch, then one
 * access per expert in order, slot release before slot allocation. On return
 * slots_out[i] is the slot of experts[i]; hit_out[i] (optional) its hit bit,
 * evicted_out[i] (optional) the expert evicted by that access or -1. */
int gx_policy_serve(gx_policy * policy, uint32_t layer, const int32_t * experts, uint32_t count,
                    int32_t * slots_out, uint8_t * hit_out, int32_t * evicted_out, gx_serve_stats * stats);
/* Slot of a resident expert, -1 otherwise (ExpertStore::slot_of). */
int32_t gx_policy_slot_of(const gx_policy * policy, uint32_t layer, uint32_t expert);
/* Cumulative counters (ExpertCache::hits/accesses/cold_bytes). */
int gx_policy_counters(const gx_policy * policy, uint64_t * hits, uint64_t * accesses, uint64_t * cold_bytes);

/* ------------------------------------------------------------- cache plan
 * Per-layer quotas from measured miss curves (CachePlan and plan_layer_quotas,
 * src/h4/h4-cache-plan.hpp:55-117, src/h4/h4-cache-plan.cpp:31-223).
 * gx_cache_plan_load reads the reference's plan file ("galactus-cache-plan 1",
 * arch/first_layer/last_layer/experts/used/source/tokens, one "curve <layer>
 * m_0 ... m_experts" line per layer, "end"); malformed files are rejected.
 * gx_plan_layer_quotas: curves [n_layers][curve_len] (misses at quota
 * 0..curve_len-1), record_bytes [n_layers] -> quotas [n_layers], never above
 * budget_bytes, never below floor or above ceiling (the reference allocator).
 * gx_policy_plan_quotas: the quotas the engine applies for a plan: the budget
 * the uniform quota buys and floor = uniform probation + 1
 * (src/h4/h4-expert-cache.cpp:136-200). GX_ERR_STATE when the plan does not
 * apply (other geometry, full residency, a result below 2 slots): keep the
 * uniform quota. The result feeds gx_arena_config.plan_quotas. */
typedef struct gx_cache_plan gx_cache_plan;
int gx_cache_plan_load(const char * path, gx_cache_plan ** plan);
void gx_cache_plan_destroy(gx_cache_plan * plan);
int gx_cache_plan_info(const gx_cache_plan * plan, uint32_t * first_layer, uint32_t * last_layer, uint32_t * experts,
                       uint32_t * used, char * arch, size_t arch_cap);
int gx_cache_plan_curve(const gx_cache_plan * plan, uint32_t layer, uint32_t * misses);
int gx_plan_layer_quotas(const uint32_t * curves, uint32_t n_layers, uint32_t curve_len, const uint64_t * record_bytes,
                         uint64_t budget_bytes, uint32_t floor, uint32_t ceiling, uint32_t * quotas);
int gx_policy_plan_quotas(const gx_profile * profile, uint64_t capacity_bytes, double protected_fraction,
                          const gx_cache_plan * plan, uint32_t * quotas);

/* ------------------------------------------------------------------ arena
 * The slot arena in HBM (one slab per layer, quota x record bytes, 16 KiB
 * aligned) and the pinned host tier that backs it (every record of every
 * layer, record layout down | gate | up). Replaces ExpertStore's arena and
 * DualVolumeReader's SSD reads (src/h4/h4-expert-store.cpp:29-90,
 * src/h4/h4-reader.cpp:284-305). */
typedef struct gx_arena gx_arena;

typedef struct gx_arena_config {
    gx_profile profile;
    uint64_t capacity_bytes;
    double protected_fraction;   /* GALACTUS_H4_PROTECTED; 0.75 in the reference */
    int policy;                  /* GX_POLICY_* */
    const uint32_t * plan_quotas;/* optional */
    int device;
    int host_tier;               /* 1: allocate the pinned host tier (all records) */
    int64_t max_tokens;          /* largest micro-batch the layer entry point will see */
    int64_t hidden;              /* H, for the layer entry point's scratch */
    int64_t intermediate;        /* I */
    void * host_tier_base;       /* optional caller-owned PINNED tier (layer-major, expert-minor records,
                                    record_bytes apart); used instead of allocating one when host_tier = 1 */
} gx_arena_config;

int gx_arena_create(const gx_arena_config * config, gx_arena ** out);
int gx_arena_destroy(gx_arena * arena);
/* Pinned host copy of record (layer, expert): fill it before the first serve. */
void * gx_arena_host_record(gx_arena * arena, uint32_t layer, uint32_t expert);
/* Copy one record into the host tier (the pack reader's job in the reference). */
int gx_load_record(gx_arena * arena, uint32_t layer, uint32_t expert, const void * src, uint64_t bytes);
/* Device base of a layer's slab, its record stride and slot count: the three
 * expert tensors of the layer are views at base + role offset with
 * nb[2] = record (create_exps, diff:2293-2296). */
int gx_arena_layer_view(gx_arena * arena, uint32_t layer, void ** base, uint64_t * record_bytes, uint32_t * slots);
gx_policy * gx_arena_policy(gx_arena * arena);
/* Number of keys currently resident with valid bytes in HBM for a layer. */

/* The remap node (galactus_h4::remap_ids, diff:2146-2150; strided read and
 * write of scripts/derive-remap-strides.py:30-75). Reads expert ids from a
 * host I32 tensor [ne0, ne1] with byte strides nb0, nb1, serves the layer
 * (policy, then one host->HBM copy per miss on the arena's copy stream), and
 * writes slot ids into a host I32 tensor with byte strides dnb0, dnb1.
 * `stream` (the consumer's stream) is made to wait for the copies, and the
 * copies wait for everything already queued on `stream`. */
int gx_remap_serve(gx_arena * arena, uint32_t layer,
                   const int32_t * ids, int64_t ne0, int64_t ne1, int64_t nb0, int64_t nb1,
                   int32_t * slots, int64_t dnb0, int64_t dnb1,
                   void * stream, gx_serve_stats * stats);

/* Copy the bytes of one slot back to host memory, after every copy queued so
 * far has landed (the slot-content audit of src/h4/h4-serve-check.cpp:63-91). */
int gx_arena_read_slot(gx_arena * arena, uint32_t layer, uint32_t slot, void * dst, uint64_t bytes);

/* Serve every expert of every layer once (full-residency warm-up), copies included. */
int gx_arena_warm_all(gx_arena * arena, void * stream);

typedef struct gx_arena_stats {
    uint64_t serves;
    uint64_t hits;
    uint64_t misses;
    uint64_t evictions;
    uint64_t bytes_h2d;
    uint64_t copies;
} gx_arena_stats;
int gx_stats(gx_arena * arena, gx_arena_stats * stats);

/* Kernel timing of the layer entry point: when enabled, every call records
 * CUDA events around its two kernels on the caller's stream; read returns the
 * summed device milliseconds of the gate/up and down kernels and the number of
 * calls since the last read (waiting for the last event). */
int gx_arena_timing(gx_arena * arena, int enable);
int gx_arena_timing_read(gx_arena * arena, double * gate_up_ms, double * down_ms, uint64_t * calls);

/* ---------------------------------------------------------------- kernels
 * ggml_mul_mat_id with ggml's tensor conventions (all device pointers):
 *   as   expert weights, row r of expert e at as + e*nb02 + r*nb01, ne00 x ne01 per expert
 *   b    f32 [ne00, ne11, ne12] with byte strides nb11, nb12 (ne11 is 1 or k)
 *   ids  i32 [ne20 = k, ne21 = T] with byte stride nbi1 between tokens
 *   dst  f32 [ne01, k, T] contiguous
 * The f32 activations are quantized to the weight type's vec_dot_type inside
 * the kernel (Q8_0 for Q8_0/MXFP4, Q8_K otherwise) and every output is the
 * CPU's vec_dot of the quantized row, bit for bit (diff:335-345, 1049-1054,
 * 1167-1174, 1254-1259, 1366-1370). Requires ne00 % 64 == 0 (Q8_0 family)
 * or % 256 == 0 (Q8_K family), 16-byte aligned as/nb01*tile/nb02. */
int gx_mul_mat_id(int type, const void * as, int64_t ne00, int64_t ne01, int64_t nb01, int64_t nb02, int64_t n_as,
                  const float * b, int64_t ne11, int64_t ne12, int64_t nb11, int64_t nb12,
                  const int32_t * ids, int64_t ne20, int64_t ne21, int64_t nbi1,
                  float * dst, void * stream);

/* Activation quantization alone (quantize_row_q8_0 / quantize_row_q8_K):
 * rows of ne0 f32 at src + i*nb1 -> blocks at dst + i*dst_row_stride. */
int gx_quantize_rows(int vec_dot_type, const float * src, int64_t ne0, int64_t nrows, int64_t nb1,
                     void * dst, int64_t dst_row_stride, void * stream);

/* out = silu(g) * u, silu(x) = x / (1 + exp(-x)) */
int gx_swiglu(const float * g, const float * u, float * out, int64_t n, void * stream);
/* out = min(g,limit) / (1 + exp(alpha * -min(g,limit))) * (clamp(u,-limit,limit) + 1) */
int gx_swiglu_oai(const float * g, const float * u, float * out, int64_t n, float alpha, float limit, void * stream);
/* out[h,t] = sum over s = 0..k-1, in order, of w[s,t] * y[h,s,t] (one rounding per product and per add) */
int gx_combine(const float * y, const float * w, float * out, int64_t H, int64_t k, int64_t T, void * stream);
/* The library's exp, elementwise (the one SiLU uses) */
int gx_expf(const float * x, float * y, int64_t n, void * stream);

/* ------------------------------------------------------------- MoE layer
 * One routed-expert FFN layer, end to end on the device:
 *   remap (policy + miss copies) -> gate/up mul_mat_id + activation
 *   -> down mul_mat_id -> weighted combine in slot order.
 * x: device f32 [H, T]; ids: HOST i32 [k, T] (contiguous); w: device f32 [k, T];
 * out: device f32 [H, T]. Record layout down | gate | up (offsets below).
 * A micro-batch whose distinct experts exceed the policy's batch bound
 * min(quota, probation) (the reference's micro-batch rule,
 * src/h4/h4-expert-cache.cpp:105-124) runs in expert-major waves of at most
 * that many experts; the output bits do not depend on the wave schedule. */
typedef struct gx_layer_desc {
    int32_t type_gate;
    int32_t type_up;
    int32_t type_down;
    int32_t act;        /* GX_ACT_* */
    float alpha;        /* SWIGLU_OAI */
    float limit;        /* SWIGLU_OAI */
    int64_t hidden;     /* H */
    int64_t intermediate; /* I */
    uint64_t off_gate;  /* byte offset of gate inside a record (down at 0) */
    uint64_t off_up;
} gx_layer_desc;

int gx_moe_layer_forward(gx_arena * arena, uint32_t layer, const gx_layer_desc * desc,
                         const float * x, const int32_t * ids, const float * w, int64_t k, int64_t T,
                         float * out, void * stream, gx_serve_stats * stats);

/* The shared expert of a layer (DeepSeek-style MoE: one dense FFN every token
 * runs with weight 1 beside the routed experts): one record in the routed
 * layout (down | gate | up at desc's offsets), resident in device memory and
 * owned by the caller. */
typedef struct gx_shared_expert {
    const void * record;      /* device address of the record */
    gx_layer_desc desc;       /* its types (e.g. Q4_K), hidden = the layer's H, intermediate, offsets */
} gx_shared_expert;

/* gx_moe_layer_forward plus the shared expert: out = moe_out + shexp(x), the
 * ggml_add(moe_out, ffn_shexp) that follows build_moe_ffn in upstream
 * llama.cpp (the tail the routed output feeds, diff:2153-2191); shexp is
 * silu(x W_gate) * (x W_up) W_down with ggml's mul_mat order per row.
 * The shared intermediate may not exceed k * the routed intermediate. */
int gx_moe_layer_forward_shared(gx_arena * arena, uint32_t layer, const gx_layer_desc * desc,
                                const float * x, const int32_t * ids, const float * w, int64_t k, int64_t T,
                                const gx_shared_expert * shared, float * out, void * stream,
                                gx_serve_stats * stats);

/* A stack of consecutive MoE layers for one micro-batch whose routes are all
 * known (the reference's "token" serving regime, src/h4/h4-expert-store.hpp:
 * 13-16): for each layer i, layer first_layer+i runs as gx_moe_layer_forward
 * on x[i], ids + i*k*T, w[i] -> out[i]. x, w, out are arrays of n_layers
 * device pointers; ids is HOST i32 [n_layers, T, k]. Stats are summed. */
int gx_moe_stack_forward(gx_arena * arena, uint32_t first_layer, uint32_t n_layers, const gx_layer_desc * desc,
                         const float * const * x, const int32_t * ids, const float * const * w, int64_t k, int64_t T,
                         float * const * out, void * stream, gx_serve_stats * stats);

/* A captured decode plan for a stack of layers, recorded once in a CUDA graph
 * with fixed input, weight and output pointers and slot ids read from a
 * device array. Each run serves every layer through the policy on the host
 * (misses copied as in gx_moe_layer_forward), copies the slot ids to the
 * device and launches the graph. Same results as gx_moe_stack_forward.
 *
 * For decode sizes (k*T <= 64) and the weight-type pairs Q8_0/Q8_0,
 * Q4_K/Q6_K, MXFP4/MXFP4 and IQ1_S/IQ1_S the graph holds ONE persistent
 * cooperative kernel for all layers, which streams the expert rows of the
 * whole stack through a bulk-copy ring with no drain between layers (it needs
 * every layer's slot ids when it starts, which the plan's run provides).
 * Otherwise, or with GX_PLAN_LAYERWISE, the graph holds the three kernels of
 * every layer.
 *
 * flags: GX_PLAN_TIMING records CUDA events around the kernels (layerwise
 * plans then run without programmatic overlap); gx_stack_plan_timing returns
 * the summed gate/up and down kernel milliseconds of the last run, or, for
 * the stack kernel, its whole duration in gate_up_ms and 0 in down_ms.
 * No reference counterpart: the reference has no device graph. */
#define GX_PLAN_TIMING 1
#define GX_PLAN_LAYERWISE 2
typedef struct gx_stack_plan gx_stack_plan;
typedef struct gx_stack_plan_info {
    int32_t stack_kernel;     /* 1: one persistent kernel for the stack, 0: three kernels per layer */
    int32_t grid;             /* CTAs of the stack kernel */
    int32_t threads;          /* threads per CTA */
    int32_t ctas_per_sm;
    int32_t stages;           /* bulk-copy ring stages per CTA (tensor_cores 2: TMA ring stages) */
    int32_t rows_gate_up;     /* gate (and up) rows per gate/up unit */
    int32_t rows_down;        /* down rows per expert per down unit */
    uint32_t smem_bytes;      /* dynamic shared memory per CTA */
    int32_t tensor_cores;     /* where the block dots of MXFP4 jobs run: 2 on the tensor cores (tcgen05
                                 kind::f8f6f4) fed by TMA from the plan's copy of the slots in a
                                 tensor-core record layout (the default for k = 4 stacks whose copies
                                 fit in free device memory; the copy follows the arena's fills), 1 on
                                 the tensor cores with CUDA-core repacking (GX_STACK_MMA=1), 0 on the
                                 CUDA cores (GX_STACK_MMA=0, and every other stack) */
} gx_stack_plan_info;
int gx_stack_plan_create(gx_arena * arena, uint32_t first_layer, uint32_t n_layers, const gx_layer_desc * desc,
                         const float * const * x, const float * const * w, float * const * out, int64_t k, int64_t T,
                         int flags, gx_stack_plan ** plan);
int gx_stack_plan_run(gx_stack_plan * plan, const int32_t * ids, void * stream, gx_serve_stats * stats);
int gx_stack_plan_timing(gx_stack_plan * plan, double * gate_up_ms, double * down_ms);
int gx_stack_plan_info_get(const gx_stack_plan * plan, gx_stack_plan_info * info);
int gx_stack_plan_destroy(gx_stack_plan * plan);

/* ---------------------------------------------------------- no allocation
 * One routed-expert FFN layer (gate/up + activation, down + weighted combine)
 * that allocates nothing, for callers that may not call cudaMalloc: a host
 * framework that owns every device allocation through its own pool, a plugin
 * loaded into such a process, or a path that cannot absorb an allocation's
 * latency and synchronization. The caller passes the expert records (slot 0's
 * record at slot0_record, record_bytes apart, n_slots of them, roles at the
 * offsets of desc), the layer input x [T, H] (device), HOST slot ids [T, k],
 * router weights w [T, k] (device) and out [T, H] (device); results equal
 * gx_moe_layer_forward's for the same slots.
 * Scratch is one fixed __device__ array of GX_NOALLOC_SCRATCH_BYTES inside
 * the library, held by every GPU that loads it until exit; k*T, H and I above
 * the GX_NOALLOC_MAX_* limits are rejected with GX_ERR_INVALID. Every call on
 * a device shares the array: calls that overlap on the GPU race and must be
 * serialized by the caller. Each call outside a stream capture looks up the
 * array's address on its device; a call inside a capture uses the address of
 * the last call outside one (make one first; after a reset of the device's
 * context, make another before capturing again).
 * No counterpart in the reference. */
#define GX_NOALLOC_MAX_PAIRS 64
#define GX_NOALLOC_MAX_HIDDEN 8192
#define GX_NOALLOC_MAX_INTERMEDIATE 4096
#define GX_NOALLOC_SCRATCH_BYTES (2u * 1024u * 1024u)
int gx_moe_ffn_noalloc(const gx_layer_desc * desc, const void * slot0_record, uint64_t record_bytes, uint32_t n_slots,
                       const float * x, const int32_t * slots, const float * w, int64_t k, int64_t T, float * out,
                       void * stream);

/* ------------------------------------------------------------ GGUF tier
 * Routed-expert weights read from a GGUF checkpoint (version 2/3): the
 * blk.L.ffn_{down,gate,up}_exps.weight tensors ([ne0, ne1, n_expert], expert
 * e's rows contiguous) give the record of (L, e) as down | gate | up, the
 * layout of the reference's packs and profile (scripts/moe-profile.py:116-211,
 * records padded to 16 KiB). gx_gguf_moe_info reads the geometry;
 * gx_arena_load_gguf copies every record of the arena's layers into its host
 * tier (as gx_load_record). gx_fnv1a64 is the record fingerprint of the
 * reference's paranoia check (scripts/verify-paranoia-trace.py:8-20). */
typedef struct gx_gguf_moe {
    char arch[64];
    uint32_t first_layer, last_layer, experts, used, block_count;
    uint32_t type_gate, type_up, type_down;
    uint64_t hidden, intermediate;
    uint64_t record_bytes, record_bytes_raw;
} gx_gguf_moe;
int gx_gguf_moe_info(const char * path, gx_gguf_moe * info);
int gx_arena_load_gguf(gx_arena * arena, const char * path, uint32_t * records_loaded);
uint64_t gx_fnv1a64(const void * data, uint64_t n);

/* --------------------------------------------------------------- router
 * The step before the routed-expert FFN, on the device: router logits
 * [rows, n_expert] (rows = n_layers * T, layer-major) to the selected expert
 * ids [rows, k] and their weights [rows, k], as upstream llama.cpp's
 * build_moe_ffn computes them at the reference's pinned commit
 * (patches/UPSTREAM-COMMIT.txt; the selection is the view the remap node
 * receives, patches/galactus-h4-llamacpp.diff:2124-2150, docs/STUDY.md:74):
 *   gating    SOFTMAX: probs = soft_max(logits); SIGMOID: probs = 1/(1+e^-x);
 *             SOFTMAX_WEIGHT: probs = logits, softmax over the k weights;
 *   bias      selection scores = probs + bias[layer] (bias may be NULL);
 *   groups    n_groups > 1: the n_group_used groups with the largest sum of
 *             their two best scores keep theirs, the others get -inf;
 *   top-k     the k best selection scores, best first (a tie goes to the
 *             lower expert id);
 *   weights   probs at the selected ids; then SOFTMAX_WEIGHT's softmax; norm_w
 *             divides by max(sum, 2^-14); scale_w multiplies by w_scale.
 * Softmax is ggml's arm64 CPU order (exp of x - max, float sums of four
 * consecutive values accumulated in double, times (float)(1/sum)), with the
 * library's own expf; the oracle restates it bit for bit. slot_table
 * [n_layers, n_expert] (device, or NULL) also maps each id to its slot
 * (gx_arena_slot_table writes it; -1 = not resident, reported through the
 * device error word). Limits: 1 <= k <= 32, k <= n_expert <= 1024,
 * n_groups <= 32 with n_expert % n_groups == 0, at least two experts per group
 * and n_group_used * n_expert / n_groups >= k. Logits must be finite. */
#define GX_GATING_SOFTMAX 0
#define GX_GATING_SIGMOID 1
#define GX_GATING_SOFTMAX_WEIGHT 2
typedef struct gx_router_desc {
    int32_t gating;
    int32_t n_expert;
    int32_t n_expert_used;
    int32_t n_groups;       /* <= 1: no group-limited selection */
    int32_t n_group_used;
    int32_t norm_w;
    int32_t scale_w;
    float w_scale;
} gx_router_desc;
/* logits: device f32, row stride ld elements; bias: device f32 [n_layers,
 * n_expert] or NULL; ids/weights (and slots when slot_table is given): device
 * [n_layers * T, k]. */
int gx_router_forward(const gx_router_desc * desc, const float * logits, int64_t ld, const float * bias, int64_t T,
                      int64_t n_layers, int32_t * ids, float * weights, const int32_t * slot_table, int32_t * slots,
                      void * stream);
/* The current slot of every expert of layers [first_layer, first_layer +
 * n_layers), or -1, written to table (device i32 [n_layers, n_expert]) on
 * the stream. Returns GX_ERR_STATE if a layer has a non-resident expert and
 * require_all is set. */
int gx_arena_slot_table(gx_arena * arena, uint32_t first_layer, uint32_t n_layers, int32_t * table, int require_all,
                        void * stream);
/* A stack plan routed on the device: the router writes the plan's ids, slots
 * and weights (the plan's weight pointers must be consecutive [T, k] slices
 * of one buffer, w[i] = w[0] + i*T*k), then the plan's graph runs; no host
 * round trip. Every layer of the plan must be pinned (all of its experts
 * resident, which holds for good once it does: a layer whose quota covers
 * all experts never evicts), otherwise GX_ERR_STATE. stats counts every pair
 * a hit. With a route trace open, the ids are read back after the step and
 * recorded. ids_out (device i32 [n_layers * T, k] or NULL) receives the ids. */
int gx_stack_plan_run_routed(gx_stack_plan * plan, const gx_router_desc * desc, const float * logits, int64_t ld,
                             const float * bias, int32_t * ids_out, void * stream, gx_serve_stats * stats);

/* ---------------------------------------------------------- route trace
 * The route observer of the reference (src/h4/h4-route-observer.hpp:58-304):
 * every micro-batch served through an arena or a policy (layer, tokens, k,
 * the expert ids in order, each with its residency bit sampled before the
 * serve, the serve's clock and the host->HBM bytes it issued) is buffered in
 * memory and written once, in the reference's "galactus.route-observer.v1"
 * text format, at gx_route_observer_close or at exit. Also opened by
 * GALACTUS_H4_ROUTES=<file> (GALACTUS_H4_ROUTES_CAP caps the entries), read at
 * the first serve. Observational only: nothing it does changes a slot. */
int gx_route_observer_open(const char * path, const char * arch, uint64_t entry_cap);
int gx_route_observer_close(void);

/* ------------------------------------------------------- expert parallel
 * The experts of a model shard over G ranks, one process per GPU: expert e
 * lives on rank e % G (GX_EP_MODULO) or e / ceil(E/G) (GX_EP_BLOCK), where
 * its local id is e / G, respectively e - rank*ceil(E/G). Each rank owns an
 * arena over its local experts (created as usual, with n_expert = the local
 * count and max_tokens >= the pairs it may receive per layer). A layer step
 * for the rank's own T tokens:
 *   dispatch   every (token, slot) pair sends the token's input row and the
 *              global expert id to the expert's rank (NCCL send/recv, one
 *              group per step; pairs of local experts stay local);
 *   compute    the received pairs run the routed-expert FFN on the local
 *              arena (remap with local ids, gate/up, activation, down) with
 *              one slot each and unit router weight, i.e. the bare down
 *              output of each pair;
 *   combine    each pair's output row goes back to its home rank, which
 *              sums w[t,s]*y[t,s] in slot order s = 0..k-1 (the single-GPU
 *              combine, so results are bit-identical to one GPU holding all
 *              experts).
 * nccl_comm is an ncclComm_t of the caller covering exactly the G ranks with
 * this rank numbering (e.g. the communicator of torch's NCCL process group);
 * the library calls ncclGroupStart/End, ncclSend and ncclRecv from the NCCL
 * already loaded in the process (or libnccl.so.2, or GX_NCCL_LIB).
 * gx_ep_plan is the host-only routing step: the pairs this rank sends to each
 * peer, in (token, slot) order grouped by destination rank.
 * No counterpart in the reference (it runs on one machine). */
#define GX_EP_MODULO 0
#define GX_EP_BLOCK 1
typedef struct gx_ep gx_ep;
int gx_ep_owner(int32_t placement, uint32_t n_expert, int32_t world, int32_t expert, int32_t * rank, int32_t * local_id);
int gx_ep_plan(int32_t placement, uint32_t n_expert, int32_t world, const int32_t * ids, int64_t k, int64_t T,
               int32_t * send_counts, int32_t * send_pairs);
int gx_ep_init(gx_arena * local_arena, void * nccl_comm, int32_t rank, int32_t world, uint32_t n_expert,
               int32_t placement, gx_ep ** ep);
int gx_ep_destroy(gx_ep * ep);
/* dispatch: x device f32 [T, H]; ids HOST i32 [T, k] of global expert ids.
 * Synchronizes the stream twice: the ranks' shapes and statuses (a call one
 * rank rejects fails on every rank), then the peers' pair counts and expert
 * ids (needed on the host for the slot policy). */
int gx_ep_dispatch(gx_ep * ep, uint32_t layer, const float * x, const int32_t * ids, int64_t k, int64_t T, int64_t H,
                   void * stream);
/* compute: the pairs received by the last dispatch, on the local arena */
int gx_ep_compute(gx_ep * ep, const gx_layer_desc * desc, void * stream, gx_serve_stats * stats);
/* combine: w device f32 [T, k] router weights, out device f32 [T, H] */
int gx_ep_combine(gx_ep * ep, const float * w, float * out, void * stream);
/* the three in sequence */
int gx_ep_layer_forward(gx_ep * ep, uint32_t layer, const gx_layer_desc * desc, const float * x, const int32_t * ids,
                        const float * w, int64_t k, int64_t T, float * out, void * stream, gx_serve_stats * stats);
/* n_layers consecutive layers whose routes are all known (the stack regime of
 * gx_moe_stack_forward) in one step: x, w, out arrays of n_layers device
 * pointers ([T, H], [T, k], [T, H]); ids HOST i32 [n_layers, T, k] of global
 * expert ids. Two host synchronizations per step (the shape and id headers,
 * whatever n_layers), one row exchange and one result exchange for all
 * layers; the owners compute layer by layer without synchronizing. Every rank
 * must pass the same first_layer, n_layers, k and H; T may differ. A call one
 * rank rejects fails on every rank before any row moves. */
int gx_ep_stack_forward(gx_ep * ep, uint32_t first_layer, uint32_t n_layers, const gx_layer_desc * desc,
                        const float * const * x, const int32_t * ids, const float * const * w, int64_t k, int64_t T,
                        float * const * out, void * stream, gx_serve_stats * stats);

/* ------------------------------------------------------------- synthetic
 * Seeded synthetic data written straight into device memory (test and bench
 * inputs; the same generator is restated in the oracle):
 *   gx_synth_normal: f32 ~ N(0, sigma) (4-term Irwin-Hall), element i of stream (seed, stream_id)
 *   gx_synth_weights: n_rows rows of ne00 elements of `type`, quantized from
 *     N(0, sigma) (Q8_0, Q4_K, Q6_K) or uniform over codes (MXFP4, IQ1_S) */
int gx_synth_normal(float * dst, int64_t n, uint64_t seed, uint64_t stream_id, float sigma, void * stream);
int gx_synth_weights(int type, void * dst, int64_t ne00, int64_t n_rows, uint64_t seed, uint64_t stream_id,
                     float sigma, void * stream);

#ifdef __cplusplus
}
#endif

#endif /* GALACTUS_B200_H */
