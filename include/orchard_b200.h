/*
 * orchard_b200.h -- C ABI of liborchard_b200.so, the B200 (sm_100a) implementation of
 * Orchard's quantised Llama-layer path.
 *
 * Conventions
 *   - Every function returns ORCH_OK (0) or a nonzero ORCH_ERR_* status; the message of
 *     the last failure on the calling thread is orch_last_error().
 *   - Pointers are device pointers unless stated; sizes are element counts unless stated.
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream).
 *     Compute calls only enqueue work; orch_d2h/orch_sync wait.
 *   - Activation dtype codes follow the reference's DType enum order
 *     (src/runtime/tensor.h:11-15): ORCH_F32 = Float32, ORCH_F16 = Float16.
 *   - The packed INT4 format is the reference's (orchard/quantizer.py:3-78):
 *     uint8 [N, K/2] (low nibble = even k) + fp16 scales [N, K/32], value (q-8)*scale.
 *
 * Each surface entry point cites the reference interface it replaces: the
 * MetalBackend method (src/platform/metal_backend.h) and its pybind11 binding
 * (src/bindings.cpp).
 */
#ifndef ORCHARD_B200_H
#define ORCHARD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ORCH_OK = 0,
  ORCH_ERR_INVALID = 1,        /* bad argument: null pointer, size, alignment, shape */
  ORCH_ERR_CUDA = 2,           /* a CUDA runtime call failed */
  ORCH_ERR_UNSUPPORTED = 3,    /* shape/dtype outside what the kernels implement */
  ORCH_ERR_NOT_INITIALIZED = 4,
  ORCH_ERR_TIMEOUT = 5,        /* a bounded device wait ran out */
  ORCH_ERR_DEVICE_CHECK = 6    /* a kernel's own bounds check rejected an input */
};

enum { ORCH_F32 = 0, ORCH_F16 = 1 };

/* ---- library / device ---------------------------------------------------------------- */
int orch_version(void);
const char* orch_status_string(int status);
const char* orch_last_error(void);

/* MetalBackend::initialize (metal_backend.h:14; bindings.cpp:16). Selects `device` and
 * prepares kernel attributes. `resource_path` is accepted for signature parity (the
 * reference compiles .metal sources found there at run time); kernels here are compiled
 * ahead of time, so a non-NULL path must only name an existing directory. */
int orch_init(int device, const char* resource_path);
/* MetalBackend::is_available (metal_backend.h:15; bindings.cpp:17). 1 if a device is usable. */
int orch_is_available(void);
/* MetalBackend::get_device_name (metal_backend.h:16; bindings.cpp:18). */
int orch_device_name(char* buf, size_t len);
/* Reads and clears the device-side check flags: nonzero after a kernel rejected an input and
 * skipped the work it covers. Bits: 1 a Q/K/V row's position outside the cache or RoPE
 * table (that row's q/k/v not written); 2 an attention row's position outside the cache
 * or a bad prefill unit (its output not written); 4 an embedding id outside the vocabulary
 * (zero row); 8 a cache slot outside [0, num_slots) (no cache read or write for that row);
 * 256 a tensor-core GEMM's bounded wait ran out; 512 a peer all-reduce's wait for another
 * rank ran out. Covers the allocation-free attention entry point's flags as well. */
int orch_device_check(uint32_t* flags_out, void* stream);

/* ---- buffers (metal_backend.h:19-22; tensor.cpp:17-72) -------------------------------- */
int orch_alloc(size_t bytes, void** ptr);                                   /* create_buffer   */
int orch_free(void* ptr);                                                   /* release_buffer  */
int orch_h2d(void* dst, const void* host_src, size_t bytes, void* stream);  /* copy_to_buffer  */
int orch_d2h(void* host_dst, const void* src, size_t bytes, void* stream);  /* copy_from_buffer (synchronises) */
int orch_memset(void* dst, int value, size_t bytes, void* stream);
int orch_sync(void* stream);

/* ---- reference operator surface (half activations, as the Metal kernels) -------------- */
/* run_matmul (metal_backend.h:25-26; bindings.cpp:20-22): fp32 C[M,N] = A[M,K] B[K,N]. */
int orch_matmul(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                void* stream);
/* run_matmul_simd (metal_backend.h:29-30; bindings.cpp:23-25): fp16 in/out, fp32 accumulate. */
int orch_matmul_simd(const void* a, const void* b, void* c, uint32_t M, uint32_t N, uint32_t K,
                     void* stream);
/* run_rmsnorm (metal_backend.h:32; bindings.cpp:26-28): rows of N, `count` rows. */
int orch_rmsnorm(const void* in, const void* weight, void* out, float eps, uint32_t N,
                 uint32_t count, void* stream);
/* run_rope (metal_backend.h:33-34; bindings.cpp:29-31): in/out [seq_len, num_heads, head_dim],
 * cos/sin [seq_len, head_dim/2]; interleaved pairs, each row its own angles. */
int orch_rope(const void* in, const void* cos, const void* sin, void* out, uint32_t head_dim,
              uint32_t num_heads, uint32_t seq_len, void* stream);
/* run_gemv_q8_0 (metal_backend.h:36-37; bindings.cpp:32-34): int8 [N,K] + fp16 [N,K/32]. */
int orch_gemv_q8_0(const void* w, const void* scales, const void* in, void* out, uint32_t K,
                   uint32_t N, void* stream);
/* run_gemv_q4_0 (metal_backend.h:39-40; bindings.cpp:35-37). */
int orch_gemv_q4_0(const void* w, const void* scales, const void* in, void* out, uint32_t K,
                   uint32_t N, void* stream);
/* run_gemm_q4_0 (metal_backend.h:42-43; bindings.cpp:38-40): in [B,K] -> out [B,N], with the
 * quantizer's nibble order (the reference batched kernel's pairing defect is not replicated). */
int orch_gemm_q4_0(const void* w, const void* scales, const void* in, void* out, uint32_t K,
                   uint32_t N, uint32_t B, void* stream);
/* run_add / run_mul / run_silu (metal_backend.h:46-48; bindings.cpp:41-49). */
int orch_add(const void* a, const void* b, void* c, uint32_t size, void* stream);
int orch_mul(const void* a, const void* b, void* c, uint32_t size, void* stream);
int orch_silu(const void* in, void* out, uint32_t size, void* stream);
/* run_softmax (metal_backend.h:49; bindings.cpp:50-52): row softmax of [rows, cols]. */
int orch_softmax(const void* in, void* out, uint32_t rows, uint32_t cols, void* stream);
/* run_embedding (metal_backend.h:50; bindings.cpp:53-55): int32 ids -> fp16 rows. `vocab` is
 * added so out-of-range ids are rejected (zero rows + device check flag) instead of read. */
int orch_embedding(const void* ids, const void* weights, void* out, uint32_t num_tokens,
                   uint32_t hidden_dim, uint32_t vocab, void* stream);

/* ---- dtype-explicit forms of the surface (the reference host allocates Float32
 *      activations, orchard/model.py:86-92; these serve Tensor dtypes exactly) ----------- */
int orch_rmsnorm_ex(const void* in, int in_dt, const void* weight, int w_dt, void* out,
                    int out_dt, float eps, uint32_t N, uint32_t count, void* stream);
int orch_rope_ex(const void* in, int in_dt, const void* cos, const void* sin, int tab_dt,
                 void* out, int out_dt, uint32_t head_dim, uint32_t num_heads,
                 uint32_t seq_len, void* stream);
int orch_gemm_q4_0_ex(const void* w, const void* scales, const void* in, int in_dt, void* out,
                      int out_dt, uint32_t K, uint32_t N, uint32_t B, void* stream);
int orch_gemm_q8_0_ex(const void* w, const void* scales, const void* in, int in_dt, void* out,
                      int out_dt, uint32_t K, uint32_t N, uint32_t B, void* stream);
/* op: 0 add, 1 mul */
int orch_binary_ex(int op, const void* a, const void* b, void* c, int dt, uint32_t size,
                   void* stream);
int orch_silu_ex(const void* in, void* out, int dt, uint32_t size, void* stream);
/* SwiGLU in one pass, out = silu(gate) * up (orchard/model.py:179-180, which runs run_silu
 * then run_mul, elementwise.metal:13-30): fp32 arithmetic, one rounding to dt on store. */
int orch_swiglu_ex(const void* gate, const void* up, void* out, int dt, uint32_t size,
                   void* stream);
int orch_softmax_ex(const void* in, int in_dt, void* out, int out_dt, uint32_t rows,
                    uint32_t cols, void* stream);
int orch_embedding_ex(const void* ids, const void* weights, int w_dt, void* out, int out_dt,
                      uint32_t num_tokens, uint32_t hidden_dim, uint32_t vocab, void* stream);

/* ---- on-device packers, bit-identical to the host packers ----------------------------- */
/* quantize_q4_0 (orchard/quantizer.py:3-78) of w [N,K] (w_dt F32 or F16), group 32. */
int orch_quantize_q4_0(const void* w, int w_dt, void* packed, void* scales, uint32_t N,
                       uint32_t K, void* stream);
/* INT8 per output channel: int8 [N,K] + fp16 [N] (the BASELINE sweep's INT8 format;
 * rounding rule of the reference's C++ packer, src/main.cpp:35-64). */
int orch_quantize_q8_pc(const void* w, int w_dt, void* q, void* scales, uint32_t N, uint32_t K,
                        void* stream);
/* INT8 group-32 (src/main.cpp:35-64). */
int orch_quantize_q8_0(const void* w, int w_dt, void* q, void* scales, uint32_t N, uint32_t K,
                       void* stream);

/* INT8 per-channel skinny GEMM: out[b,n] = s[n] * sum_k q[n,k] in[b,k]. */
int orch_gemm_q8_pc(const void* w, const void* scales, const void* in, int in_dt, void* out,
                    int out_dt, uint32_t K, uint32_t N, uint32_t B, void* stream);

/* ---- fused decode path (additive; the reference runs these steps as separate synchronous
 *      ops plus host attention, orchard/model.py:78-195) -------------------------------- */
/* LoRA on the fused projections (orchard/model.py:60-76: out += (x.A).B, B pre-scaled by
 * alpha/r). A projection with R output regions (q/k/v: 3, gate/up: 2, others: 1) takes
 * lora_t fp32 [M, R, r] = x.A (orch_lora_xa) and lora_b fp32 [R, r, width]; the delta is
 * added to the accumulator before the epilogue. lora_t == NULL disables it. */
int orch_lora_xa(const void* x, const float* a, float* t, uint32_t M, uint32_t K, uint32_t R,
                 void* stream);
/* x fp16 [M,K] -> resid fp32 [M,N] += W x   (O-proj / down-proj + residual add,
 * orchard/model.py:147-157,184-193). */
int orch_q4_linear_resid(const void* w, const void* scales, const void* x, float* resid,
                         uint32_t M, uint32_t K, uint32_t N, const float* lora_t,
                         const float* lora_b, uint32_t lora_r, void* stream);
/* Gate/up + SwiGLU (orchard/model.py:167-180). w13: [2F, K] with gate and up rows
 * interleaved in blocks of 16 (rows 32b..32b+15 = gate 16b.., 32b+16.. = up 16b..);
 * h fp16 [M,F] = silu(gate) * up. */
int orch_q4_linear_swiglu(const void* w13, const void* s13, const void* x, void* h, uint32_t M,
                          uint32_t K, uint32_t F, const float* lora_t, const float* lora_b,
                          uint32_t lora_r, void* stream);
/* Q/K/V projection + RoPE + KV-cache append (orchard/model.py:94-124). wqkv: [3H, K] =
 * [Wq; Wk; Wv]. Rotates q and k with cos/sin tables [max_pos, head_dim/2] (fp32) at
 * pos[m]; writes q fp16 [M,H]; appends k, v fp16 to the caches laid out
 * [num_slots][num_heads][max_seq][head_dim] at slot slots[m] (NULL = m), position pos[m];
 * a row whose slot is outside [0, num_slots) or whose position is outside the cache writes
 * nothing and sets a device check bit (8 / 1). H = num_heads * head_dim must be below 65536
 * and head_dim even. */
int orch_q4_qkv_rope(const void* wqkv, const void* sqkv, const void* x, uint32_t M, uint32_t K,
                     uint32_t H, uint32_t num_heads, const int32_t* pos, const int32_t* slots,
                     const float* cos_tab, const float* sin_tab, uint32_t max_pos, void* q_out,
                     void* k_cache, void* v_cache, uint32_t max_seq, uint32_t num_slots,
                     const float* lora_t, const float* lora_b, uint32_t lora_r, void* stream);
/* Tiled INT4 weights (no reference counterpart: the engine's device copy of a weight
 * packed by orchard/quantizer.py:3-78, re-laid once at load). Rows in tiles of 128, k in
 * blocks of 256, each (tile, block) one contiguous 18 KB run of packed nibbles and scales,
 * zero-padded; orch_q4t_bytes() gives the size. orch_q4t_pack converts a reference-layout
 * weight [N, K/2] + scales [N, K/32]. The orch_q4t_* GEMMs take the tiled buffer in place of
 * (w, scales) and otherwise match orch_gemm_q4_0_ex (fp16 activations) and the fused
 * entry points above; they always run on the tcgen05 tensor-core kernel. */
size_t orch_q4t_bytes(uint32_t N, uint32_t K);
int orch_q4t_pack(const void* packed, const void* scales, uint32_t N, uint32_t K, void* tiled,
                  void* stream);
int orch_q4t_gemm(const void* tiled, const void* in, void* out, int out_dt, uint32_t K, uint32_t N,
                  uint32_t M, void* stream);
int orch_q4t_linear_resid(const void* tiled, const void* x, float* resid, uint32_t M, uint32_t K,
                          uint32_t N, const float* lora_t, const float* lora_b, uint32_t lora_r,
                          void* stream);
int orch_q4t_linear_swiglu(const void* tiled13, const void* x, void* h, uint32_t M, uint32_t K,
                           uint32_t F, const float* lora_t, const float* lora_b, uint32_t lora_r,
                           void* stream);
int orch_q4t_qkv_rope(const void* tiled_qkv, const void* x, uint32_t M, uint32_t K, uint32_t H,
                      uint32_t num_heads, const int32_t* pos, const int32_t* slots,
                      const float* cos_tab, const float* sin_tab, uint32_t max_pos, void* q_out,
                      void* k_cache, void* v_cache, uint32_t max_seq, uint32_t num_slots,
                      const float* lora_t, const float* lora_b, uint32_t lora_r, void* stream);
/* RMSNorm fused in front of the tiled Q/K/V (+ RoPE + KV append) and gate/up (+ SwiGLU)
 * projections: the reference's rms_norm -> projection pair (orchard/model.py:86-101,160-172;
 * orchard/kernels/rmsnorm.metal:23-35). x is the fp32 residual [M, K], norm_w fp32 [K] (both
 * 16-byte aligned); the activations are fp16(x * rsqrt(sum(x^2) / K + eps) * norm_w). Up to 8
 * rows, the GEMV computes the norm itself (one launch; xn is not written); with more rows the
 * normalised rows go to the fp16 scratch xn [M, K] and the tensor-core GEMM reads them. No
 * LoRA term (its x.A needs xn first: use orch_rmsnorm_ex and the unfused entry points). */
int orch_q4t_rms_qkv_rope(const void* tiled_qkv, const float* x, const float* norm_w, float eps,
                          void* xn, uint32_t M, uint32_t K, uint32_t H, uint32_t num_heads,
                          const int32_t* pos, const int32_t* slots, const float* cos_tab,
                          const float* sin_tab, uint32_t max_pos, void* q_out, void* k_cache,
                          void* v_cache, uint32_t max_seq, uint32_t num_slots, void* stream);
int orch_q4t_rms_linear_swiglu(const void* tiled13, const float* x, const float* norm_w, float eps,
                               void* xn, void* h, uint32_t M, uint32_t K, uint32_t F, void* stream);
/* Rows up to which the orch_q4t_* entry points take the GEMV (8; ORCHARD_GEMV_MAX_M in the
 * environment may lower it); above it they run on the tcgen05 tensor-core GEMM. */
uint32_t orch_gemv_max_rows(void);
/* Decode attention over the device KV cache (orchard/model.py:117-137): for each row m and
 * head h, softmax(q.K[0..pos] / sqrt(hd)) . V[0..pos]. q, out fp16 [M, num_heads*head_dim].
 * The caches hold num_slots slots; row m reads slot slots[m] (NULL = m). A row whose slot
 * is outside [0, num_slots) or whose position is outside [0, max_seq) reads nothing, is not
 * written, and sets device check bit 8 / 2. Long rows are split over positions; the split
 * partials go to `workspace` (fp32, orch_attention_workspace_bytes() bytes). */
size_t orch_attention_workspace_bytes(uint32_t M, uint32_t num_heads, uint32_t head_dim,
                                      uint32_t max_seq);
int orch_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                          const int32_t* pos, const int32_t* slots, void* out, uint32_t M,
                          uint32_t num_heads, uint32_t head_dim, uint32_t max_seq,
                          uint32_t num_slots, void* workspace, size_t workspace_bytes,
                          void* stream);
/* INT4 GEMMs with fp16 activations and at least `m` rows run on the tcgen05 tensor-core
 * kernel (TMEM accumulators, TMA-fed activations); fewer rows use the mma.sync decode
 * kernel. 0 disables the tensor-core kernel. Default 17 (ORCHARD_TC_MIN_M overrides). */
int orch_set_tc_min_m(uint32_t m);
/* Causal attention for a prefill chunk (no counterpart in the reference, whose prefill
 * attention is the per-token host loop of orchard/model.py:112-144). q and out are [M, heads,
 * 128] fp16, the caches as for orch_attention_decode. `units` (device, 16-byte aligned) lists
 * num_units records of four int32 (row0, rows, slot, pos0): rows row0 .. row0 + rows - 1
 * (1..64 of them) belong to cache slot `slot` at positions pos0, pos0 + 1, ..., and their
 * K/V are already in the cache; each row attends to positions 0..its own. Rows in no unit are
 * not written; a unit whose slot is outside [0, num_slots) is skipped and sets device check
 * bit 8. Tensor-core kernel: head_dim 128 only (ORCH_ERR_UNSUPPORTED otherwise). */
int orch_attention_prefill(const void* q, const void* k_cache, const void* v_cache, const int32_t* units,
                           uint32_t num_units, void* out, uint32_t M, uint32_t num_heads, uint32_t head_dim,
                           uint32_t max_seq, uint32_t num_slots, void* stream);
/* Batched-decode INT4 GEMMs on tiled weights (orch_q4t_*, 9..64 activation rows): mode 0
 * (default) always uses the per-tile tensor-core kernel, 1 the persistent stream-K kernel
 * (work split evenly over two CTAs per SM, split tiles summed by a fix-up pass), 2 picks
 * stream-K for shapes whose tile count lands between one and one and a half waves of SMs.
 * ORCHARD_TC_SK=0/1/2 in the environment sets the initial mode. */
int orch_set_stream_k(int mode);
/* Vocabulary-split greedy sampling (no reference counterpart: the reference samples on the
 * host, orchard/model.py:244-252). orch_argmax_pairs writes, per row of a logits slice
 * [M, V] whose first column is vocabulary id `base`, the pair (max logit, base + argmax)
 * as floats; orch_argmax_merge reduces the all-gathered pairs [world][B][2] of rows
 * row0 .. row0 + rows - 1 to token ids: the highest logit, the lowest id among equal
 * logits, a NaN first (np.argmax over the whole vocabulary). */
int orch_argmax_pairs(const float* logits, uint32_t M, uint32_t V, uint32_t base, float* pairs,
                      void* stream);
int orch_argmax_merge(const float* pairs, uint32_t world, uint32_t B, uint32_t row0, uint32_t rows,
                      int32_t* tok, void* stream);
/* Temperature sampling on the device, replacing the host sampler of orchard/model.py:244-252:
 * per row of logits [M, V] (fp32), p = softmax((l - max) / T) in fp32, and the token is the
 * first id whose running sum of p exceeds uniforms[row] (the inverse CDF that
 * np.random.choice evaluates with its one uniform draw; the caller draws the uniforms from
 * its own RNG, so the NumPy stream of the reference can be followed). */
int orch_sample_rows(const float* logits, uint32_t M, uint32_t V, float temperature,
                     const float* uniforms, int32_t* tok, void* stream);
/* Decode attention that allocates nothing (no counterpart in the reference). Same inputs,
 * outputs and arithmetic as orch_attention_decode, but the split-position partials live in
 * a 1 MiB array inside the library (orch_attention_noalloc_max_bytes()) that every GPU
 * loading the library keeps until the process exits. For callers that cannot allocate
 * device memory: hosts capturing CUDA graphs of their own, memory-static real-time hosts,
 * plugin hosts that pass only the call's tensors. The first call on a device looks up the
 * array's device address; make it before any stream capture on that device. A shape whose
 * partials exceed the array fails with ORCH_ERR_UNSUPPORTED. Every call on a device uses the
 * same array and leaves its partials there; each call writes every partial it reads, so no
 * clearing is needed, but calls whose execution overlaps on one GPU (for example on two
 * streams) race and must be ordered by the caller. Rows rejected by the position or slot
 * check set their bits in a flag word that also lives inside the library; orch_device_check
 * reports it. */
size_t orch_attention_noalloc_max_bytes(void);
int orch_attention_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                  const int32_t* pos, const int32_t* slots, void* out,
                                  uint32_t M, uint32_t num_heads, uint32_t head_dim,
                                  uint32_t max_seq, uint32_t num_slots, void* stream);
/* Row argmax of fp32 logits [M, V] (first index of the maximum, as np.argmax;
 * orchard/model.py:244-246). */
int orch_argmax_rows(const float* logits, uint32_t M, uint32_t V, int32_t* out, void* stream);
/* Gathers fp32 residual rows x[m] = table[ids[m]] (table fp16 or fp32 [V, H]). */
int orch_embed_rows(const int32_t* ids, const void* table, int table_dt, float* x, uint32_t M,
                    uint32_t H, uint32_t V, void* stream);

/* ---- peer-memory all-reduce of the head split ------------------------------------------
 * The reference runs on one device (orchard/model.py:78-195 has no collective); the head
 * split's order of operations (orchard_b200/parallel.py: attention_head_split,
 * ffn_head_split) sums the fp32 residual over the ranks after the O and the down
 * projections. One process per GPU of one box. Each rank allocates a region of
 * orch_peer_region_bytes(world, max_floats) bytes (orch_alloc), zeroes it, exports it with
 * orch_ipc_handle (64 bytes), and opens every other rank's handle with orch_ipc_open; after
 * a barrier (so no rank writes into a region before it is zeroed) orch_peer_allreduce sums
 * x[0..n) over the ranks in place: bases[q] is rank q's region as mapped here (own included),
 * the same world and max_floats the regions were sized with; n <= max_floats, both multiples
 * of 4; every rank makes the same calls in the same order. The result is the same bits on
 * every rank (slots added in rank order). algo 1: one shot (every rank sends its whole buffer
 * to every rank, 8 n (world - 1) bytes out); 2: two shots (reduce-scatter then all-gather,
 * 16 n (world - 1) / world bytes out, one more NVLink crossing); 0: one shot on two ranks or
 * while it sends at most 1 MiB, two shots otherwise. A wait for a peer that runs out (~5 s)
 * sets device check bit 512. Regions and mappings live until orch_ipc_close / orch_free. */
size_t orch_peer_region_bytes(uint32_t world, uint32_t max_floats);
int orch_ipc_handle(void* base, void* handle_out);
int orch_ipc_open(const void* handle, void** base_out);
int orch_ipc_close(void* base);
int orch_peer_allreduce(void* const* bases, uint32_t rank, uint32_t world, uint32_t max_floats,
                        float* x, uint32_t n, int algo, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ORCHARD_B200_H */
