/*
 * yskn_b200.h -- C ABI of the B200 (sm_100a) compressed-integer linear path.
 *
 * Drop-in surface for the reference's compressed linear operator (YASAKANI
 * `.yskn` weights: trellis-coded 3/4-bit codes, a 4096-pair value table and one
 * scale per row, Hadamard-512 rotations; int8 activations; exact int64 sums).
 *
 * Conventions (as the reference's include/yskn_abi.h and src/c_api.cpp:11-14):
 *   - every call returns int: 0 on success, a negative YSKN_E* code on failure;
 *     yskn_b200_last_error() gives a thread-local message for the last failure;
 *   - device pointers are caller-owned; work is ordered on the caller's CUDA
 *     stream (`void* stream`, NULL = legacy default stream) with no hidden
 *     synchronisation, except in the *_host helpers and yskn_b200_status();
 *   - the hot calls (weighted_sums, quantize, restore, linear) allocate nothing;
 *     matrix handles own their device copies, created once at load time;
 *   - one call at a time per matrix handle and stream (crates/yskn-engine/src/pool.rs:29).
 * Plain C types only: a Rust `Backend::Cuda`, Go cgo or Python ctypes binds it directly.
 */
#ifndef YSKN_B200_H
#define YSKN_B200_H
#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define YSKN_B200_API __declspec(dllexport)
#else
#define YSKN_B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define YSKN_OK 0
#define YSKN_EINVAL (-1)      /* bad shape, pointer or argument (reference: -1)            */
#define YSKN_ECUDA (-2)       /* a CUDA runtime error                                      */
#define YSKN_EOVERFLOW (-3)   /* integer accumulation exceeds i64 (compressed_linear.rs:245) */
#define YSKN_ENONFINITE (-4)  /* a non-finite activation / restored value (compressed_linear.rs:82,100,342) */
#define YSKN_ETIMEDOUT (-5)   /* a bounded device wait gave up                             */
#define YSKN_ENOMEM (-6)      /* device allocation failed (create-time only)               */

#define YSKN_LAYOUT_ROW 0     /* docs/FORMAT.md:141-151 */
#define YSKN_LAYOUT_WARP 1

#define YSKN_SIGNS_SPLITMIX64 0 /* docs/FORMAT.md:159-180 */
#define YSKN_SIGNS_MULBERRY32 1

typedef struct yskn_b200_matrix yskn_b200_matrix;
typedef struct yskn_b200_tp yskn_b200_tp;

#define YSKN_B200_TP_HANDLE_BYTES 64 /* one rank's exchange-area handle (a CUDA IPC handle) */

/* Thread-local message of the last failure (src/c_api.cpp:11-14 `yskn_last_error`). */
YSKN_B200_API const char* yskn_b200_last_error(void);

/* Synchronise `stream`, then read and clear the device-side error word that kernels
 * raise for conditions only the device sees (non-finite activations, i64 overflow,
 * timed-out waits). Returns 0 or the first YSKN_E* code raised since the last call. */
YSKN_B200_API int yskn_b200_status(void* stream);

/* Replaces include/yskn_abi.h:19 / src/repack.cu:21-26: identical permutation of
 * warp-layout code words into the reference's "frag" order; -1 unless rows%64==0
 * and wps%4==0; asynchronous on `cuda_stream`. */
YSKN_B200_API int yskn_repack_warp_to_frag(const uint32_t* d_words, uint32_t* d_frag, int rows, int seqs, int wps,
                                           void* cuda_stream);
/* Replaces include/yskn_abi.h:20 / src/repack.cu:27-32: host buffers in and out. */
YSKN_B200_API int yskn_repack_warp_to_frag_host(const uint32_t* h_words, uint32_t* h_frag, int rows, int seqs,
                                                int wps);

/* Host helper: n signs (+1/-1) at positions offset.. of the stream `rule`/`seed`
 * defines. Replaces src/signs.hpp:9-31 (crates/yskn-format/src/signs.rs:12-38). */
YSKN_B200_API int yskn_b200_signs(int rule, uint64_t seed, uint64_t offset, int64_t n, int8_t* h_out);

/* Bytes of the B200 streaming layout for a matrix (warp order, rows padded to 32). */
YSKN_B200_API int64_t yskn_b200_pack_bytes(int physical_rows, int cols, int bits);

/* Layout transform of one matrix's code words (row or warp layout, device memory)
 * into the B200 streaming layout (d_out, yskn_b200_pack_bytes() bytes). Replaces the
 * load-time reorder src/repack.cu + src/lnord.cu:58-88 (lnord_build). */
YSKN_B200_API int yskn_b200_pack(const uint32_t* d_words, int layout, int physical_rows, int cols, int bits,
                                 void* d_out, void* stream);

/* Load one compressed matrix (replaces src/loader.cpp:19-60 Model::upload_linear +
 * lnord_build; the Rust side is crates/yskn-engine/src/mapped.rs:78-186):
 *   d_codes       the tensor's code stream as stored (`layout`), in device memory;
 *   lut16_host    8192 binary16 table values; scale16_host: physical_rows binary16 scales;
 *   signs_in_host cols signs; signs_out_host physical_rows signs or NULL (no output rotation).
 * Builds the int8 table and effective row scales (compressed_linear.rs:138-158) and
 * packs the codes. Synchronous (load time). NULL on failure (see last_error). */
YSKN_B200_API yskn_b200_matrix* yskn_b200_matrix_create(const uint32_t* d_codes, int layout, int rows,
                                                        int physical_rows, int cols, int bits,
                                                        const uint16_t* lut16_host, const uint16_t* scale16_host,
                                                        const int8_t* signs_in_host, const int8_t* signs_out_host);
/* Tensor-parallel shard of the same tensor (the arguments describe the whole tensor as
 * above): physical rows [row_begin, row_end) (row_begin % 8 == 0; whole 512-row blocks
 * when there is an output rotation) and columns [col_begin, col_end) (whole 512-column
 * groups). Column-parallel projections split rows, row-parallel ones split columns; the
 * shard's sums equal the whole tensor's sums restricted to those rows / columns. No
 * counterpart function in the reference, whose engine runs on one GPU; the split
 * follows the 512-blocks of docs/FORMAT.md. */
YSKN_B200_API yskn_b200_matrix* yskn_b200_matrix_create_shard(const uint32_t* d_codes, int layout, int rows,
                                                              int physical_rows, int cols, int bits,
                                                              const uint16_t* lut16_host,
                                                              const uint16_t* scale16_host,
                                                              const int8_t* signs_in_host,
                                                              const int8_t* signs_out_host, int row_begin,
                                                              int row_end, int col_begin, int col_end);
/* A shard of several row ranges (row_ranges: n_ranges pairs begin, end; 1..16), stored
 * one after another: the handle's row i is the i-th row of the ranges in order (every
 * range but the last whole 8-row blocks of real rows; whole 512-row blocks with an output
 * rotation). One rank's rows of a projection whose parts split separately, such as the
 * query, key and value rows of in_proj_qkv for the heads the rank runs. No counterpart in
 * the reference (one GPU). */
YSKN_B200_API yskn_b200_matrix* yskn_b200_matrix_create_rows(const uint32_t* d_codes, int layout, int rows,
                                                             int physical_rows, int cols, int bits,
                                                             const uint16_t* lut16_host,
                                                             const uint16_t* scale16_host,
                                                             const int8_t* signs_in_host,
                                                             const int8_t* signs_out_host, int n_ranges,
                                                             const int* row_ranges, int col_begin, int col_end);
YSKN_B200_API void yskn_b200_matrix_destroy(yskn_b200_matrix* m);
/* rows, physical_rows, cols, bits, has_output_rotation, packed bytes. */
YSKN_B200_API int yskn_b200_matrix_info(const yskn_b200_matrix* m, int64_t* out6);
/* Device copies owned by the handle: int8 table (8192 B), effective row scales
 * (f32[physical_rows]), input signs (i8[cols]), output signs (i8[physical_rows] or NULL). */
YSKN_B200_API const int8_t* yskn_b200_matrix_lut8(const yskn_b200_matrix* m);
YSKN_B200_API const float* yskn_b200_matrix_tau(const yskn_b200_matrix* m);
YSKN_B200_API const int8_t* yskn_b200_matrix_signs_in(const yskn_b200_matrix* m);
YSKN_B200_API const int8_t* yskn_b200_matrix_signs_out(const yskn_b200_matrix* m);

/* ---- .yskn containers (docs/FORMAT.md:33-107) ------------------------------------
 * yskn_b200_file_open replaces the reference's readers, src/format.hpp:26-61
 * (Container::open) and crates/yskn-format/src/lib.rs:97-172 (Container::new) with
 * crates/yskn-format/src/tensor.rs:31-63,83-196,212-236 (descriptors): the file is
 * memory-mapped read-only and checked as the reference reader checks it (magic,
 * version, declared lengths, JSON header, every descriptor and data region, unique
 * names, zero padding). NULL on failure, with the reason in yskn_b200_last_error().
 * Opening uses no GPU. The handle and the strings it returns stay valid until
 * yskn_b200_file_close. */
typedef struct yskn_b200_file yskn_b200_file;
#define YSKN_ROLE_BODY 0
#define YSKN_ROLE_HEAD 1
#define YSKN_ROLE_EMBEDDING 2
#define YSKN_ROLE_DRAFT 3
#define YSKN_VECTOR_F16 0
#define YSKN_VECTOR_BF16 1
#define YSKN_TENSOR_INFO_FIELDS 17
YSKN_B200_API yskn_b200_file* yskn_b200_file_open(const char* path);
YSKN_B200_API void yskn_b200_file_close(yskn_b200_file* f);
/* The `model` member of the header, as its JSON text. */
YSKN_B200_API const char* yskn_b200_file_model_json(const yskn_b200_file* f);
YSKN_B200_API int yskn_b200_file_tensor_count(const yskn_b200_file* f);
YSKN_B200_API int yskn_b200_file_vector_count(const yskn_b200_file* f);
/* Index of the tensor or vector named `name` (*is_vector says which), or YSKN_EINVAL. */
YSKN_B200_API int yskn_b200_file_find(const yskn_b200_file* f, const char* name, int* is_vector);
YSKN_B200_API const char* yskn_b200_file_tensor_name(const yskn_b200_file* f, int i);
/* Tensor i's descriptor with the format's defaults applied (tensor.rs:83-196), in this
 * order: role (YSKN_ROLE_*), rows, cols, physical_rows, bits, layout (YSKN_LAYOUT_*),
 * stream_off, stream_bytes, lut_off, scale_off, input sign rule (YSKN_SIGNS_*), seed,
 * offset, has output rotation (0/1), output sign rule (-1 if none), seed, offset. */
YSKN_B200_API int yskn_b200_file_tensor_info(const yskn_b200_file* f, int i, int64_t* out17);
YSKN_B200_API const char* yskn_b200_file_vector_name(const yskn_b200_file* f, int i);
/* Vector i: offset, count, dtype (YSKN_VECTOR_*). */
YSKN_B200_API int yskn_b200_file_vector_info(const yskn_b200_file* f, int i, int64_t* out3);
/* Vector i's n values as f32 (f16 converted exactly; bf16 as the upper half of a float),
 * as crates/yskn-format/src/lib.rs reads them. */
YSKN_B200_API int yskn_b200_file_vector_read(const yskn_b200_file* f, int i, float* h_out, int64_t n);
/* Matrix handle of tensor i (replaces src/loader.cpp:19-60 Model::upload_linear): the
 * code stream goes to the device through a pinned staging buffer, the sign streams are
 * built from the tensor's rotations, then as yskn_b200_matrix_create[_shard] (the shard
 * bounds as there). Roles body, head and draft; an embedding is rejected (the reference
 * decodes it row by row with its 16-bit table). Synchronous; NULL on failure. */
YSKN_B200_API yskn_b200_matrix* yskn_b200_file_load_matrix(const yskn_b200_file* f, int i);
YSKN_B200_API yskn_b200_matrix* yskn_b200_file_load_matrix_shard(const yskn_b200_file* f, int i, int row_begin,
                                                                 int row_end, int col_begin, int col_end);

/* ---- Coded embedding rows (docs/spec/02_COMPRESSED_LINEAR.md:271-303) -------------
 * Replaces the reference's coded-embedding path, Engine35 set-up + q35_embed
 * (src/engine35.cpp:272-299, src/q35_kernels.cu:1501-1574): per token, each table's row
 * is decoded with its own binary16 table and row scale, the tables are added in order,
 * then per 512 columns H512, * 1/sqrt(512), * the main table's input signs, one rounding
 * to bf16. */
typedef struct yskn_b200_embedding yskn_b200_embedding;
/* n_parts 1..3 tables (main, then residuals) of rows x cols (cols % 512 == 0), each with
 *   d_codes[k] its code stream in row layout (docs/FORMAT.md:141-144), device memory;
 *   bits[k], lut16_host[k] (8192 binary16), scale16_host[k] (rows binary16);
 * signs_in_host: the main table's cols input signs. Copies everything (synchronous). */
YSKN_B200_API yskn_b200_embedding* yskn_b200_embedding_create(int n_parts, const uint32_t* const* d_codes,
                                                             const int* bits, int rows, int cols,
                                                             const uint16_t* const* lut16_host,
                                                             const uint16_t* const* scale16_host,
                                                             const int8_t* signs_in_host);
YSKN_B200_API void yskn_b200_embedding_destroy(yskn_b200_embedding* e);
/* d_out: bf16 bits [M][cols] (16-byte aligned) for the int32 token ids d_tokens [M].
 * A token outside 0..rows-1 gives a zero row and, from yskn_b200_status, YSKN_EINVAL. */
YSKN_B200_API int yskn_b200_embedding_lookup(const yskn_b200_embedding* e, const int32_t* d_tokens, int M,
                                             uint16_t* d_out, void* stream);
/* From a file: tensors main_i and (or -1) res_i, res2_i, checked as the reference engine
 * checks a coded embedding (src/engine35.cpp:272-299). */
YSKN_B200_API yskn_b200_embedding* yskn_b200_file_load_embedding(const yskn_b200_file* f, int main_i, int res_i,
                                                                 int res2_i);

/* Residual addition and deferred normalisation between projections (replaces the
 * residual/normalisation part of q35_res_norm_xsm_kernel, src/q35_kernels.cu:1437-1463,
 * and q35_xsm_r, :81-85; docs/spec/05_RESIDUAL_NORM_MLP.md:53-141). Per row of M:
 *   d_hidden     bf16 [M][cols], updated in place: bf16(hidden + bf16(projection));
 *   d_projection f32 [M][cols] (a restored projection output), or NULL for no addition;
 *   d_norm_weight bf16 [cols]; eps from the model header;
 *   d_input      f32 [M][cols] = hidden * (1 + weight): the next operator's x (yskn_b200_linear);
 *   d_inv_rms    f32 [M] = rsqrtf(sum of squares / cols + eps), in the reference's
 *                reduction order: the next operator's inv_rms;
 *   d_gate       bf16 [M][cols] copy of d_input, or NULL.
 * cols a multiple of 512. */
YSKN_B200_API int yskn_b200_residual_prepare(uint16_t* d_hidden, const float* d_projection,
                                             const uint16_t* d_norm_weight, int M, int cols, float eps,
                                             float* d_input, float* d_inv_rms, uint16_t* d_gate, void* stream);

/* MLP nonlinear step (replaces src/q35_kernels.cu:1402-1421; docs/spec/
 * 05_RESIDUAL_NORM_MLP.md:156-176): with g = bf16(gate), u = bf16(up),
 * d_out = bf16(bf16(g / (1 + expf(-g))) * u) as f32 [M][n], the down projection's input.
 * d_gate, d_up: the restored f32 outputs of gate_proj and up_proj. */
YSKN_B200_API int yskn_b200_gated_product(const float* d_gate, const float* d_up, int M, int n, float* d_out,
                                          void* stream);

/* Greedy token and top-8 raw logits per row of head logits (replaces the greedy and
 * top-k kernels, src/misc_kernels.cu:59-88,100-140, src/q35_sample.cu:131-178; docs/spec/
 * 06_OUTPUT_HEAD_SAMPLER.md:31-64): order (larger logit, smaller id) from (-FLT_MAX,
 * INT_MAX), so NaN and -inf are never chosen. d_logits f32 [M][n] (yskn_b200_linear of
 * the head matrix with the row's inverse RMS); d_token int32 [M]; d_top8_logits f32
 * [M][8] and d_top8_ids int32 [M][8] in that order; any output may be NULL (not all). */
YSKN_B200_API int yskn_b200_head_select(const float* d_logits, int M, int n, int32_t* d_token, float* d_top8_logits,
                                        int32_t* d_top8_ids, void* stream);
/* The head split over vocabulary rows (tensor parallelism; the reference's head runs on one
 * GPU, src/misc_kernels.cu:59-88): the greedy token and top 8 of the whole row from the
 * parts' yskn_b200_head_select top 8: part q's f32 logits and int32 ids [M][8] start
 * part_stride elements after part q - 1's (8 M when the parts are packed), its ids local to
 * it (h_id_offsets[q], a host array, is its first row's id). The order is the same, so the
 * result is bit-identical to yskn_b200_head_select over the whole row. n_parts 1..8;
 * outputs as yskn_b200_head_select's. */
YSKN_B200_API int yskn_b200_head_merge(const float* d_part_logits, const int32_t* d_part_ids, int64_t part_stride,
                                       const int32_t* h_id_offsets, int n_parts, int M, int32_t* d_token,
                                       float* d_top8_logits, int32_t* d_top8_ids, void* stream);

/* Attention inputs from the q/k/v projection outputs (replaces the head preparation of
 * the q35 attention, src/q35_kernels.cu:1013-1059 and :1091-1104, and the cache rotation
 * src/kvx_codec.cuh:11-48; docs/spec/04_ATTENTION.md:15-106): per row and head, bf16
 * projections; query and key heads normalised by their RMS times (1 + q_norm / k_norm),
 * RoPE at d_positions[row] on channels i, i+32 (i < 32); every head through the
 * 256-element cache rotation. d_q f32 [M][n_qh][512] (query, then gate channels per
 * head), d_k, d_v f32 [M][n_kvh][256]; out: d_query bf16 [M][n_qh][256] (the attention's
 * q), d_gate bf16 [M][n_qh][256] (its gate), d_k_rot, d_v_rot f32 [M][n_kvh][256] (the KV
 * encoder's rows). rsqrtf, cosf and sinf are CUDA's, as in the reference. */
YSKN_B200_API int yskn_b200_attention_prep(const float* d_q, const float* d_k, const float* d_v,
                                           const uint16_t* d_q_norm, const uint16_t* d_k_norm,
                                           const int32_t* d_positions, float eps, int M, int n_qh, int n_kvh,
                                           uint16_t* d_query, uint16_t* d_gate, float* d_k_rot, float* d_v_rot,
                                           void* stream);

/* Gated DeltaNet decode step (replaces src/q35_kernels.cu:746-820 and :864-980; docs/spec/
 * 03_GATED_DELTANET.md:33-160), ordinary causal rows. Gates: d_gates f32 [M][96] (48 b, then
 * 48 a) from the layer's weighted hidden row d_hidden (bf16 [M][hidden], the gate copy of
 * yskn_b200_residual_prepare), its d_inv_rms [M], and the dense bf16 weights d_wb, d_wa
 * [48][hidden] (hidden a multiple of 1024). Step: d_qkv f32 [M][10240] and d_z f32 [M][6144]
 * (the restored in_proj_qkv / in_proj_z outputs), the bf16 conv weights [10240][4], A_log,
 * dt_bias [48] and norm weight [128]; commits after n_commit rows (0..M; 0 = a provisional
 * verification pass): d_state f32 [48][128][128] becomes the state after row n_commit - 1 and
 * d_history bf16 [3][10240] (the newest committed projected rows, oldest first; zero at the
 * start) takes the committed rows (docs/spec/03_GATED_DELTANET.md:160-186). Writes d_out
 * f32 [M][6144], the gated output (bf16 values), out_proj's input. expf, rsqrtf and log1pf
 * are CUDA's, as in the reference. */
YSKN_B200_API int yskn_b200_gdn_gates(const uint16_t* d_hidden, const float* d_inv_rms, const uint16_t* d_wb,
                                      const uint16_t* d_wa, int M, int hidden, float* d_gates, void* stream);
YSKN_B200_API int yskn_b200_gdn_step(const float* d_qkv, const float* d_z, const float* d_gates,
                                     const uint16_t* d_conv_w, const uint16_t* d_a_log, const uint16_t* d_dt_bias,
                                     const uint16_t* d_norm_w, float eps, int M, int n_commit, float* d_state,
                                     uint16_t* d_history,
                                     float* d_out, void* stream);
/* The same two steps for a run of value heads, as one tensor-parallel rank holds them (the
 * reference runs the whole layer on one GPU, src/engine35.cpp:768-842; the split by value
 * head with its key heads is this library's). gates_heads: d_wb, d_wa the n_heads rows of
 * the run, d_gates f32 [M][2 n_heads] (b, then a). step_heads: value heads v_head0 ..
 * v_head0 + n_v_heads - 1 (value head h reads key head h / 3), with the query and key
 * channels of key heads qk_head0 .. qk_head0 + qk_channels / 128 - 1; d_qkv f32 [M][W],
 * W = 2 qk_channels + 128 n_v_heads, each row [query | key | value channels]; d_conv_w
 * bf16 [W][4]; d_history bf16 [3][W]; d_z and d_out f32 [M][128 n_v_heads]; d_a_log,
 * d_dt_bias [n_v_heads]; d_state f32 [n_v_heads][128][128]. Each head's results are the
 * whole layer's bits for that head. */
YSKN_B200_API int yskn_b200_gdn_gates_heads(const uint16_t* d_hidden, const float* d_inv_rms, const uint16_t* d_wb,
                                            const uint16_t* d_wa, int n_heads, int M, int hidden, float* d_gates,
                                            void* stream);
YSKN_B200_API int yskn_b200_gdn_step_heads(const float* d_qkv, const float* d_z, const float* d_gates,
                                           const uint16_t* d_conv_w, const uint16_t* d_a_log,
                                           const uint16_t* d_dt_bias, const uint16_t* d_norm_w, float eps, int M,
                                           int n_commit, int n_v_heads, int v_head0, int qk_head0, int qk_channels,
                                           float* d_state, uint16_t* d_history, float* d_out, void* stream);
/* The whole mixer in one launch (the reference's dense-gate and recurrence kernels,
 * src/q35_kernels.cu:746-820 and :864-980): yskn_b200_gdn_gates (here from d_hidden bf16
 * [M][hidden], d_inv_rms, d_wb, d_wa bf16 [heads][hidden], hidden a multiple of 1024) and
 * yskn_b200_gdn_step with the history update, bit-identical to the two calls; M = 1..64.
 * _heads: a run of value heads as yskn_b200_gdn_step_heads, d_wb / d_wa the run's rows.
 * One mixer launch in flight per device (its key-head arrival counters are the device's). */
YSKN_B200_API int yskn_b200_gdn_mixer(const uint16_t* d_hidden, const float* d_inv_rms, const uint16_t* d_wb,
                                      const uint16_t* d_wa, int hidden, const float* d_qkv, const float* d_z,
                                      const uint16_t* d_conv_w, const uint16_t* d_a_log, const uint16_t* d_dt_bias,
                                      const uint16_t* d_norm_w, float eps, int M, int n_commit, float* d_state,
                                      uint16_t* d_history, float* d_out, void* stream);
YSKN_B200_API int yskn_b200_gdn_mixer_heads(const uint16_t* d_hidden, const float* d_inv_rms, const uint16_t* d_wb,
                                            const uint16_t* d_wa, int hidden, const float* d_qkv, const float* d_z,
                                            const uint16_t* d_conv_w, const uint16_t* d_a_log,
                                            const uint16_t* d_dt_bias, const uint16_t* d_norm_w, float eps, int M,
                                            int n_commit, int n_v_heads, int v_head0, int qk_head0, int qk_channels,
                                            float* d_state, uint16_t* d_history, float* d_out, void* stream);

/* bf16 -> f32 copy of n values (exact): an operator's f32 input from a bf16 producer, such as
 * the attention output before o_proj (the reference quantises that bf16 vector directly,
 * docs/spec/04_ATTENTION.md; the operator here takes f32 input). No counterpart of its own
 * in the reference. */
YSKN_B200_API int yskn_b200_widen_bf16(const uint16_t* d_in, int64_t n, float* d_out, void* stream);

/* The scalar contract's portable functions (crates/yskn-ref/src/portable_math.rs:106-434)
 * as the library's kernels evaluate them, over n floats: fn YSKN_PM_EXP .. YSKN_PM_RSQRT
 * write d_y; YSKN_PM_SINCOS writes the cosine to d_y and the sine to d_y2 (0 and 0 for
 * a non-finite angle or one outside the reduction's range). The layer kernels (residual
 * normalisation, gated product, attention inputs, Gated DeltaNet, the attention's split
 * combine and gate) call exactly these, so their results equal yskn-ref's bit for bit.
 * No counterpart of its own in the reference (its CUDA engine's portable mode,
 * src/pm_math.cuh, is internal). */
#define YSKN_PM_EXP 0
#define YSKN_PM_EXP2 1
#define YSKN_PM_LOG 2
#define YSKN_PM_LOG1P 3
#define YSKN_PM_SIGMOID 4
#define YSKN_PM_SILU 5
#define YSKN_PM_SOFTPLUS 6
#define YSKN_PM_RSQRT 7
#define YSKN_PM_SINCOS 8
YSKN_B200_API int yskn_b200_portable_math(int fn, const float* d_x, int64_t n, float* d_y, float* d_y2, void* stream);

/* Exact weighted integer sums (the operator core). Replaces
 * crates/yskn-engine/src/model.rs:948-962 `Compute::weighted_sums` (bit-identical to
 * crates/yskn-ref/src/compressed_linear.rs:205-252) and the reference's launch_lnord /
 * launch_pfa / launch_q35_g6 / launch_gemv / launch_gemm (src/kernels.hpp:52-63).
 *   mats     n_mats (1..3) matrices sharing one input of `cols` columns;
 *   d_act    int8 [M][cols] row-major; d_scales int32 [M][cols/512];
 *   d_out[i] int64 [M][physical_rows_i] row-major (overwritten).
 * Any M >= 1. Returns YSKN_EOVERFLOW (synchronously detected) only for cols >= 262144. */
YSKN_B200_API int yskn_b200_weighted_sums(const yskn_b200_matrix* const* mats, int n_mats, const int8_t* d_act,
                                          const int32_t* d_scales, int M, int64_t* const* d_out, void* stream);
/* The first n_rows rows only: d_out int64 [M][n_rows] (crates/yskn-engine/src/pool.rs:227-244). */
YSKN_B200_API int yskn_b200_weighted_sums_prefix(const yskn_b200_matrix* mat, const int8_t* d_act,
                                                 const int32_t* d_scales, int M, int n_rows, int64_t* d_out,
                                                 void* stream);

/* Activation quantiser (replaces src/a8_prologue.cuh:64-81,122-133 and the fused
 * prologues of src/q35_kernels.cu:1402-1474; crates/yskn-ref/src/compressed_linear.rs:57-135):
 * x f32 [M][Kc] -> act int8 [M][Kc], alpha f32 [M][Kc/512], scales int32 [M][Kc/512],
 * row_quantum f32 [M]. Bit-exact. Non-finite inputs raise YSKN_ENONFINITE in the
 * device error word (read with yskn_b200_status). */
YSKN_B200_API int yskn_b200_quantize(const float* d_x, const int8_t* d_signs, int M, int Kc, int8_t* d_act,
                                     float* d_alpha, int32_t* d_scales, float* d_row_quantum, void* stream);

/* The integer grid of each activation row from a given maximum of its group scales
 * (compressed_linear.rs:113-128): d_scales[m][g] = rne(alpha * (2^24 / row_max[m])),
 * d_row_quantum[m] = row_max[m] * 2^-24. Tensor parallelism (row-parallel projections):
 * each rank quantises its own 512-column groups with yskn_b200_quantize, the ranks take
 * the maximum of their row maxima (an all-reduce MAX of M floats), and this call puts
 * every rank on the whole row's grid, so the int64 partial sums add up (all-reduce
 * SUM) to exactly the one-GPU sums. No counterpart in the single-GPU reference. */
YSKN_B200_API int yskn_b200_rescale(const float* d_alpha, const float* d_row_max, int M, int groups,
                                    int32_t* d_scales, float* d_row_quantum, void* stream);

/* Tensor-parallel row-parallel operator in one launch per rank (no counterpart in the
 * single-GPU reference; replaces quantize + all-reduce MAX + rescale + weighted_sums +
 * all-reduce SUM + restore). Each rank (one process per GPU) creates an exchange area
 * sized for its largest row-parallel matrix and gets a YSKN_B200_TP_HANDLE_BYTES handle;
 * the ranks swap handles (any host channel), then connect, which maps the peers' areas
 * over NVLink. yskn_b200_linear_rowpar then computes, on every rank, the whole output
 * of the matrix from this rank's 512-column groups: row maxima and int64 sums of
 * finished 512-row blocks go to the peers' areas with plain stores and flag words
 * (bounded waits: a peer that never arrives gives YSKN_ETIMEDOUT from
 * yskn_b200_status), and y is bit-identical to one GPU's yskn_b200_linear.
 * Every rank issues the same calls in the same order on one stream per device; calls on
 * one exchange area never overlap. mat: a shard of whole 512-column groups (all rows),
 * with an output rotation, at most max_physical_rows rows; M = 1..16; d_x_local: this
 * rank's columns of the input (f32 [M][cols of the shard]); d_y: f32 [M][rows]. */
YSKN_B200_API yskn_b200_tp* yskn_b200_tp_create(int world, int rank, int max_physical_rows, void* ipc_handle_out);
YSKN_B200_API int yskn_b200_tp_connect(yskn_b200_tp* tp, const void* handles /* world x 64 bytes, rank order */);
YSKN_B200_API void yskn_b200_tp_destroy(yskn_b200_tp* tp);
/* No counterpart in the reference. For one process that drives several GPUs (one
 * thread per device, peer access enabled): this rank's exchange area as a device
 * pointer, and a connect that takes the peers' areas as device pointers reachable from
 * this rank's device (world entries in rank order; this rank's own entry is ignored),
 * instead of IPC handles. A pointer of a rank that never runs its launches is allowed:
 * this rank's waits on it then end with YSKN_ETIMEDOUT. */
YSKN_B200_API void* yskn_b200_tp_area(yskn_b200_tp* tp);
YSKN_B200_API int yskn_b200_tp_connect_peers(yskn_b200_tp* tp, void* const* peer_areas);
/* No counterpart in the reference. Limit of each wait phase of yskn_b200_linear_rowpar
 * on the peers (the row maxima, then the block sums), in seconds at the device's
 * maximum SM clock; default 1 s, accepted 1e-6 .. 60. One deadline covers a whole
 * phase of a CTA and a timeout ends the CTA's later waits at once, so a launch whose
 * peer never arrives ends within about two limits with YSKN_ETIMEDOUT. */
YSKN_B200_API int yskn_b200_tp_set_wait(yskn_b200_tp* tp, double seconds);
YSKN_B200_API int yskn_b200_linear_rowpar(yskn_b200_tp* tp, const yskn_b200_matrix* mat, const float* d_x_local, int M,
                                          const float* d_inv_rms, float* d_y, void* stream);
/* The row-parallel operator with the residual epilogue of yskn_b200_linear_residual (the
 * reference's FIN epilogue, src/lnord.cu:119-170, and q35_res_norm_xsm_kernel,
 * src/q35_kernels.cu:1427-1474, which run on one GPU): this rank's columns of the input,
 * as f32 d_x_local [M][cols of the shard] or as int8 d_act_local with group scales
 * d_alpha_local [M][cols / 512] (exactly one; the int8 form is the local output of
 * yskn_b200_gated_product_q8); every rank updates the whole residual stream d_hidden and
 * writes the whole next input (d_act_out, d_alpha_out, d_bss_out, d_gate_out as in
 * yskn_b200_linear_residual), bit-identical to one GPU's yskn_b200_linear_residual. The
 * matrix's rows are a multiple of 512 (physical rows = rows). */
/* The row-parallel operator from this rank's int8 input columns d_act_local [M][cols of the
 * shard] with group scales d_alpha_local (the local output of yskn_b200_gated_product_q8),
 * the whole output d_y f32 [M][rows] on every rank, bit-identical to one GPU's
 * yskn_b200_linear_q8 (no counterpart in the reference, whose engine runs on one GPU). */
YSKN_B200_API int yskn_b200_linear_rowpar_q8(yskn_b200_tp* tp, const yskn_b200_matrix* mat, const int8_t* d_act_local,
                                             const float* d_alpha_local, int M, float* d_y, void* stream);
YSKN_B200_API int yskn_b200_linear_rowpar_residual(yskn_b200_tp* tp, const yskn_b200_matrix* mat,
                                                   const float* d_x_local, const int8_t* d_act_local,
                                                   const float* d_alpha_local, int M, uint16_t* d_hidden,
                                                   const uint16_t* d_norm_weight, const int8_t* d_next_signs,
                                                   int8_t* d_act_out, float* d_alpha_out, float* d_bss_out,
                                                   uint16_t* d_gate_out, void* stream);

/* The per-layer chain between projections in the operators themselves (replaces the
 * reference's fused epilogue/prologue kernels: the FIN restore of src/lnord.cu:119-170 and
 * q35_res_norm_xsm_kernel, src/q35_kernels.cu:1402-1474, which restore a projection, add it
 * to the residual stream, normalise and quantise the next operator's input in one pass;
 * scalar order residual_norm_mlp.rs:14-61,120-156 and compressed_linear.rs:57-135).
 *
 * yskn_b200_linear_residual: the whole operator of ONE matrix with an output rotation whose
 * rows (a multiple of 512, physical rows = rows) are added to the residual stream: from an
 * f32 input d_x [M][cols] or an int8 input d_act [M][cols] with group scales d_alpha
 * [M][cols/512] (exactly one of the two), it updates d_hidden (bf16 [M][rows]) to
 * bf16(h + bf16(y)) and writes the next projection's input: d_act_out int8 [M][rows] and
 * d_alpha_out [M][rows/512] (the quantiser of compressed_linear.rs:57-112 applied to
 * h * (1 + w) with d_norm_weight bf16 [rows] and the next matrix's input signs
 * d_next_signs), d_bss_out [M][rows/512] (each 512-block's sum of squares of h in the
 * spec's order) and, if d_gate_out, the bf16 copy of h * (1 + w) (the dense gates' input).
 * yskn_b200_linear_q8: the whole operator of up to 3 matrices from such an int8 input; with
 * d_bss it forms each row's 1/rms = rsqrt(sum of the block sums / cols + eps) and uses it in
 * the restore (and stores it to d_inv_rms_out if given).
 * yskn_b200_gated_product_q8: the MLP product of yskn_b200_gated_product quantised at once
 * for the down projection (its input signs d_signs): d_act int8 [M][n], d_alpha [M][n/512].
 * All three give bit for bit what the separate calls (restore, residual_prepare, quantize)
 * give; decode shapes only (M = 1..16 with the input in shared memory). */
YSKN_B200_API int yskn_b200_linear_residual(const yskn_b200_matrix* mat, const float* d_x, const int8_t* d_act,
                                            const float* d_alpha, int M, uint16_t* d_hidden,
                                            const uint16_t* d_norm_weight, const int8_t* d_next_signs,
                                            int8_t* d_act_out, float* d_alpha_out, float* d_bss_out,
                                            uint16_t* d_gate_out, void* stream);
YSKN_B200_API int yskn_b200_linear_q8(const yskn_b200_matrix* const* mats, int n_mats, const int8_t* d_act,
                                      const float* d_alpha, const float* d_bss, float eps, int M, float* d_inv_rms_out,
                                      float* const* d_y, void* stream);
YSKN_B200_API int yskn_b200_gated_product_q8(const float* d_gate, const float* d_up, int M, int n,
                                             const int8_t* d_signs, int8_t* d_act, float* d_alpha, void* stream);
/* The same chain with the residual step at the start of the NEXT operator instead of the
 * end of the previous one (replaces the same reference epilogue, src/q35_kernels.cu:1427-1474;
 * scalar order as above): the operator of up to 3 matrices sharing one input, whose input
 * is formed in the launch from the previous projection's restored rows d_y_prev f32 [M][cols]:
 * h = bf16(h_in + bf16(y)) (d_hidden_in bf16 [M][cols]), x = h * (1 + w) (d_norm_weight
 * bf16 [cols]), quantised with the matrices' input signs, 1/rms = rsqrt(sum of the block
 * sums of squares / cols + eps) applied in the restore. It stores h to d_hidden_out (another
 * buffer than d_hidden_in), and if given the bf16 copy of x to d_gate_out and 1/rms to
 * d_inv_rms_out; d_y[i] f32 [M][rows_i] as yskn_b200_linear. Bit-identical to
 * yskn_b200_residual_prepare followed by yskn_b200_linear. The previous projection restores
 * in its own launch (yskn_b200_linear / _q8 / _rowpar), so no launch ends with a serial
 * residual step. Decode shapes only (M = 1..16). */
YSKN_B200_API int yskn_b200_linear_from_residual(const yskn_b200_matrix* const* mats, int n_mats, const float* d_y_prev,
                                                 const uint16_t* d_hidden_in, uint16_t* d_hidden_out,
                                                 const uint16_t* d_norm_weight, float eps, int M, uint16_t* d_gate_out,
                                                 float* d_inv_rms_out, float* const* d_y, void* stream);

/* Restore + output rotation (replaces src/a8_prologue.cuh:10-15 xsum_combine and the
 * restore part of src/q35_kernels.cu:1402-1474; compressed_linear.rs:288-370):
 * y[m][r] = f32(ws)*row_quantum[m] (*inv_rms[m]) *tau[r]; then, if rotate_out, per
 * 512-row block H512, *0.0441941738, *s_out. d_inv_rms may be NULL. d_y f32 [M][n_rows].
 * If clear_ws != 0 the consumed int64 accumulators are zeroed (the reference clears
 * its shared accumulator when it consumes it). */
YSKN_B200_API int yskn_b200_restore(int64_t* d_ws, const float* d_row_quantum, const float* d_inv_rms,
                                    const yskn_b200_matrix* mat, int M, int rotate_out, int n_rows, int clear_ws,
                                    float* d_y, void* stream);

/* No counterpart in the reference. Same contract and results as
 * yskn_b200_weighted_sums, for callers that must not have the library allocate
 * device memory (a serving process that gave nearly all HBM to its own pool at
 * start-up, or a latency-critical loop in which cudaMalloc/cudaFree could
 * synchronise the device). It always runs the decode GEMV and keeps its
 * reduction scratch in a static device array of 5,373,952 bytes, which every GPU
 * that loads the library holds until exit. Limits (else YSKN_EINVAL): M <= 64,
 * at most 262,144 physical rows over the call's matrices, cols < 262,144.
 * All calls on a device share that array: calls that overlap on the GPU race, so
 * issue them in order on one stream. The first call on each device looks up the
 * array's device address; make that first call before any stream capture. */
YSKN_B200_API int yskn_b200_weighted_sums_noalloc(const yskn_b200_matrix* const* mats, int n_mats,
                                                  const int8_t* d_act, const int32_t* d_scales, int M,
                                                  int64_t* const* d_out, void* stream);

/* Whole operator for up to 3 matrices sharing one input: quantise x with the first
 * matrix's input signs, weighted sums, restore (with each matrix's output rotation
 * if it has one). Replaces CompressedLinear::project (compressed_linear.rs:254-285)
 * and Engine35::gemv + its post step (src/engine35.cpp:403-430).
 * d_work: caller scratch of yskn_b200_linear_work_bytes(mats, n_mats, M) bytes. */
YSKN_B200_API int64_t yskn_b200_linear_work_bytes(const yskn_b200_matrix* const* mats, int n_mats, int M);
YSKN_B200_API int yskn_b200_linear(const yskn_b200_matrix* const* mats, int n_mats, const float* d_x, int M,
                                   const float* d_inv_rms, void* d_work, float* const* d_y, void* stream);

/* Quantised-KV decode attention over packed 4-bit trellis rows, with the split
 * combination, inverse cache rotation and output gate. Replaces launch_q35_atx_pk
 * (src/q35_atxpk.cu:702-741) followed by q35_combine_kernel (src/q35_kernels.cu:
 * 1279-1399); scalar semantics Attention::output_head_with (crates/yskn-ref/src/
 * attention.rs:486-518) with the prefix schedule of attention.rs:207-232.
 *   d_q, d_gate: bf16 [M][n_query_heads][256] (queries cache-rotated; gate may be NULL,
 *     then the output is the rounded inverse-rotated head).
 *   d_k_rows, d_v_rows: u32 [n_kv_heads][capacity][8*kb], MSB-first kb-bit fields
 *     (kv_codec.rs:447-458); d_k_scales, d_v_scales: f32 [n_kv_heads][capacity].
 *   d_k_codebook, d_v_codebook: bf16 [n_kv_heads][256], bfloat(reconstruction(state));
 *   d_v_mean: f32 [n_kv_heads][256] or NULL.
 * Query row m sees cache rows [0, length - M + m]; the last is its own row. Query head
 * j reads KV head j / (n_query_heads / n_kv_heads). n_splits 0 = the reference
 * schedule (31 splits below 4096 rows, else 42); 1..64 fixed; -1 = as many splits as
 * fill one wave of the device's SMs (results differ from other split counts only by
 * float rounding). kb must be 4. All device pointers 16-byte aligned. One launch: the
 * last CTA of each (query row, KV head) combines the splits, counting arrivals in a
 * static device array of 4096 counters that the launch leaves at zero; so M *
 * n_kv_heads <= 4096, and calls on one device must not overlap (issue them in order
 * on one stream, as a decode loop does). Launched as a programmatic dependent of the
 * previous kernel on the stream: the codebooks and the cache rows before the call's M new
 * rows are read before it waits for that kernel, so that kernel must not write them (it
 * may write the M new rows, the queries and the gate).
 * d_attended: optional f32 [M][n_query_heads][256] (before the inverse rotation).
 * d_out: bf16 [M][n_query_heads][256]. d_work: yskn_b200_kv4_attention_work_bytes(). */
YSKN_B200_API int64_t yskn_b200_kv4_attention_work_bytes(int M, int n_query_heads, int length, int n_splits);
YSKN_B200_API int yskn_b200_kv4_attention(const uint16_t* d_q, const uint16_t* d_gate, const uint32_t* d_k_rows,
                                          const float* d_k_scales, const uint32_t* d_v_rows,
                                          const float* d_v_scales, const uint16_t* d_k_codebook,
                                          const uint16_t* d_v_codebook, const float* d_v_mean, int M,
                                          int n_query_heads, int n_kv_heads, int length, int capacity, int kb,
                                          int n_splits, void* d_work, float* d_attended, uint16_t* d_out,
                                          void* stream);

/* Quantised-KV row encoder for packed (trellis) rows: replaces launch_tb_fast ->
 * tbf_vit_kernel / tbf2_vit_kernel + tbf_sel_kernel (src/kvq_fast.cuh:150-249,
 * src/kvq_vit2.cuh:217); scalar spec encode_packed (crates/yskn-ref/src/kv_codec.rs:
 * 408-441) for groups that are packable (mode 0, no guard, no basis; kv_profile.rs:
 * 251-286). Bit-identical words and scales.
 *   d_rows: f32 [n_rows][256] cache-rotated rows; d_row_group: i32 [n_rows] profile
 *     group of each row (layer, head, side); d_tables: i16 [n_groups][256] table codes
 *     of each group's trellis table; d_gains: f32 [n_groups] that table's gain;
 *   d_means: f32 [n_groups][256] decoded group means, or NULL; d_has_mean: u8 [n_groups]
 *     (NULL: every group has a mean when d_means is given);
 *   d_mults: f32 [n_mult] the profile's scale multipliers (1..16); kb: 4 or 5 (the
 *     profile's packed bits); vit2: the profile is vit2-eligible (kv_profile.rs:276-286).
 *   d_dest: i64 [n_rows] destination row of each encoded row in d_words / d_scales
 *     (for example head * capacity + position), or NULL for row i.
 *   d_words: u32 [*][8*kb] MSB-first fields; d_scales: f32 [*].
 * A row whose arithmetic overflows i32 or turns non-finite (the reference's Err) is not
 * written and raises YSKN_ENONFINITE at the next yskn_b200_status(). One launch, no
 * scratch: one CTA per row runs the chains of up to four multipliers at once. */
YSKN_B200_API int yskn_b200_kv_encode(const float* d_rows, const int32_t* d_row_group, int n_rows,
                                      const int16_t* d_tables, const float* d_gains, const float* d_means,
                                      const uint8_t* d_has_mean, const float* d_mults, int n_mult, int kb,
                                      int vit2, const int64_t* d_dest, uint32_t* d_words, float* d_scales,
                                      void* stream);

#ifdef __cplusplus
}
#endif
#endif /* YSKN_B200_H */
