/* Exported C ABI of libtdb.so (the framework's native sm_100a library).
 *
 * Every entry point takes raw device pointers plus a cudaStream_t passed as
 * `void* stream` and returns a CUDA error code (0 on success); the text of the
 * last host-side validation error is available from tdb_last_error().  The
 * sources include this header (through common.cuh), so the compiler checks
 * each definition against the prototype here; the Python ctypes signatures
 * are checked against it by tests/test_abi_header.py.
 *
 * ABI version: tdb_abi_version() (bumped when a prototype changes).
 */
#ifndef TDB_H_
#define TDB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- runtime (runtime.cu) ---------------------------------------------- */
int tdb_abi_version(void);
long long tdb_launch_count(void);
const char* tdb_last_error(void);
const char* tdb_error_string(int code);
int tdb_read_status(int* out4);
int tdb_clear_status(void);
int tdb_diagnostic_delay(unsigned long long cycles, void* stream);
int tdb_sm_count(int device);
int tdb_set_grid_limit(int ctas);

/* ---- symmetric memory (symm.cu) ----------------------------------------- */
int tdb_symm_handle_bytes(void);
int tdb_symm_alloc(size_t bytes, void** ptr, void* handle_out);
int tdb_symm_open(const void* handle, void** ptr);
int tdb_symm_close(void* ptr);
int tdb_symm_free(void* ptr);
int tdb_memset_async(void* ptr, int value, size_t bytes, void* stream);
int tdb_memcpy_async(void* dst, const void* src, size_t bytes, void* stream);
int tdb_can_access_peer(int device, int peer);

/* ---- TACO codec (codec.cu) ---------------------------------------------- */
int tdb_taco_encode(const void* input, void* packet, int64_t elements, void* stream);
int tdb_taco_decode(const void* packet, void* output, int64_t elements, void* stream);
int tdb_taco_reduce(const void* local, const void* remote, void* output, int64_t elements, int rank, int world,
                    void* stream);
int tdb_e4m3_probe(const float* in, uint8_t* codes, float* decoded, int64_t n, void* stream);
int tdb_taco_block_stats(const void* input, int64_t block_elements, int blocks, double* out, void* stream);

/* ---- GEMMs (gemm.cu, gemm_mx.cu) ----------------------------------------- */
int tdb_gemm_pick_tile(int M, int N, int K, int sms);
int tdb_gemm(const void* A, int a_mn, int64_t lda, const void* B, int b_mn, int64_t ldb, void* C, int64_t ldc, int M,
             int N, int K, int mode, const void* bias, const void* aux, int64_t ld_aux, void* aux_out, float alpha,
             float beta, int bn, void* stream);
long long tdb_mx_scale_bytes(long long rows, long long K);
int tdb_mx_quantize_versioned(const void* x, long long ldx, int rows, int K, void* q, void* sf, const int* version,
                              int* seen, void* stream);
int tdb_mx_quantize(const void* x, long long ldx, int rows, int K, void* q, void* sf, void* stream);
int tdb_gemm_mx(const void* A, const void* sfa, const void* B, const void* sfb, void* C, long long ldc, int M, int N,
                int K, int mode, const void* bias, void* stream);

/* ---- fused GEMM -> reduce-scatter (gemm_rs.cu) --------------------------- */
int tdb_gemm_rs(const void* A, int64_t lda, const void* B, int b_mn, int64_t ldb, int m, int N, int K, int bn,
                const int* tile_table, const uint64_t* peers, int W, int rank, int chunk_rows, uint64_t recv_off,
                uint64_t slot_bytes, uint64_t flags_off, int set, unsigned int expected, const uint8_t* qmask,
                void* out, const void* bias, const void* residual, const int* consume, int policy,
                unsigned long long* timeline, long long delay_cycles, int delay_mb, int delay_nb,
                double wait_seconds, unsigned long long* phases, const uint32_t* call_state, int quantized,
                void* stream);
int tdb_gemm_rs_mx(const void* A, int64_t lda, const void* B, int b_mn, int64_t ldb, int m, int N, int K, int bn,
                   const int* tile_table, const uint64_t* peers, int W, int rank, int chunk_rows, uint64_t recv_off,
                   uint64_t slot_bytes, uint64_t flags_off, int set, unsigned int expected, const uint8_t* qmask,
                   void* out, const void* bias, const void* residual, const int* consume, int policy,
                   unsigned long long* timeline, long long delay_cycles, int delay_mb, int delay_nb,
                   double wait_seconds, unsigned long long* phases, const uint32_t* call_state, const void* a8,
                   const void* sfa, const void* b8, const void* sfb, const uint8_t* mx_mask, void* stream);
int tdb_rs_set_variant(int variant);
int tdb_rs_advance(unsigned int* call_state, unsigned int signals, void* stream);
int tdb_gemm_rs_signals_per_block(int chunk_rows, int N, int bn);

/* ---- all-gather and fused all-gather -> GEMM (allgather.cu, ag_gemm.cu) -- */
long long tdb_ag_region_bytes(long long rows, long long cols);
int tdb_ag_prepare(const void* x, long long ldx, long long rows, long long cols, const unsigned long long* peers, int W,
                   int rank, unsigned long long heap_off, unsigned int* state, int taco, void* stream);
int tdb_allgather(const void* x, long long ldx, long long rows, long long cols, void* out,
                  const unsigned long long* peers, int W, int rank, unsigned long long heap_off, unsigned int* state,
                  double wait_seconds, void* stream);
int tdb_ag_set_variant(int variant);
int tdb_ag_gemm(const void* x, long long ldx, void* full, long long rows, int K, const void* B, int b_mn,
                long long ldb, void* C, long long ldc, int N, int mode, const void* bias, const void* aux,
                long long ld_aux, void* aux_out, float alpha, int bn, const int* tile_table,
                const unsigned long long* peers, int W, int rank, unsigned long long heap_off,
                unsigned long long region_bytes, unsigned int* state, unsigned int* ready, double wait_seconds,
                int taco, void* stream);
long long tdb_ag_gemm_region_bytes(long long rows, long long cols, int W);

/* ---- sparse vocabulary-parallel embedding exchange (embed_exchange.cu) --- */
long long tdb_embx_region_bytes(long long ml, long long H, int W);
int tdb_embx_forward(const int64_t* tokens, const void* table, long long start, long long local_vocab, const void* pos,
                     long long pos_offset, int seq, void* x, const unsigned long long* peers, int W, int rank,
                     long long ml, long long H, unsigned long long heap_off, unsigned int* state, double wait_seconds,
                     void* stream);
int tdb_embx_backward(const int64_t* tokens, const void* dy, long long ld, long long start, long long local_vocab,
                      void* out, const unsigned long long* peers, int W, int rank, long long ml, long long H,
                      unsigned long long heap_off, unsigned int* state, double wait_seconds, void* stream);

/* ---- attention (attn_tc.cu: tcgen05; attention.cu: other lengths) -------- */
int tdb_attn_fwd(const void* qkv, int64_t ld, void* out, int64_t ld_out, float* lse, int mb, int seq, int Hl,
                 float scale, void* stream);
int tdb_attn_bwd_pre(const void* out, int64_t ld_out, const void* dout, int64_t ld_dout, float* dsum, int mb, int seq,
                     int Hl, void* stream);
int tdb_attn_bwd(const void* qkv, int64_t ld, const void* out, int64_t ld_out, const void* dout, int64_t ld_dout,
                 const float* lse, float* dsum, void* dqkv, int64_t ld_dqkv, int mb, int seq, int Hl, float scale,
                 void* stream);
int tdb_attn_fwd_tc(const void* qkv, int64_t ld, void* out, int64_t ld_out, float* lse, int mb, int seq, int Hl,
                    float scale, void* stream);
int tdb_attn_fwd_tc_timeline(const void* qkv, int64_t ld, void* out, int64_t ld_out, float* lse, int mb, int seq,
                             int Hl, float scale, void* stream, unsigned long long* tl);
int tdb_attn_bwd_tc(const void* qkv, int64_t ld, const void* out, int64_t ld_out, const void* dout, int64_t ld_dout,
                    const float* lse, float* dsum, void* dqkv, int64_t ld_dqkv, int mb, int seq, int Hl, float scale,
                    void* stream);

/* ---- LayerNorm (layernorm.cu) ------------------------------------------- */
int tdb_layernorm_fwd(const void* x, const void* gamma, const void* beta, void* y, float* mean, float* rstd, int rows,
                      int H, float eps, void* stream);
int tdb_layernorm_bwd_scratch_floats(int rows, int H);
int tdb_layernorm_bwd(const void* x, const void* gamma, const float* mean, const float* rstd, const void* dy,
                      const void* dres, void* dx, float* dgamma, float* dbeta, float* partial, int rows, int H,
                      int accumulate, void* stream);
/* Allocation-free LayerNorm backward: the same computation as
 * tdb_layernorm_bwd, with the partial sums in a fixed array inside the
 * library instead of caller scratch (for callers that cannot allocate device
 * memory; see layernorm.cu).  Problems needing more than
 * tdb_layernorm_bwd_noalloc_max_floats() scratch floats are rejected; calls
 * that can overlap on one device race on the shared array. */
long long tdb_layernorm_bwd_noalloc_max_floats(void);
int tdb_layernorm_bwd_noalloc(const void* x, const void* gamma, const float* mean, const float* rstd, const void* dy,
                              const void* dres, void* dx, float* dgamma, float* dbeta, int rows, int H, int accumulate,
                              void* stream);

/* ---- elementwise, embedding, cross-entropy ------------------------------- */
int tdb_bias_residual(const void* x, const void* bias, const void* res, void* out, int64_t rows, int cols,
                      void* stream);
int tdb_colsum_scratch_floats(int rows, int cols);
int tdb_colsum(const void* x, int64_t ld, int rows, int cols, float* partial, float* out, int accumulate,
               void* stream);
int tdb_sort_tokens(const int64_t* tokens, int n, int64_t* sorted_tokens, int64_t* order, void* stream);
int tdb_embedding_fwd(const int64_t* tokens, const void* table, int64_t start, int64_t local_vocab, const void* pos,
                      int64_t pos_offset, int seq, int rows, int H, void* out, void* stream);
int tdb_add_positions(void* x, const void* pos, int64_t offset, int seq, int rows, int H, void* stream);
int tdb_embedding_bwd(const int64_t* sorted_tokens, const int64_t* sorted_rows, int rows, const void* dy,
                      int64_t start, int64_t local_vocab, int H, float* grad, void* stream);
int tdb_position_bwd(const void* dy, int rows, int64_t offset, int seq, int H, float* grad_pos, void* stream);
int tdb_xent_stats(const void* logits, int64_t ld, const int64_t* targets, int64_t vocab_start, int valid_cols,
                   int cols, int rows, float* stats, void* stream);
int tdb_xent_combine(const float* all_stats, int world, int rows, float* gstats, float* row_loss, float* loss_out,
                     float loss_scale, int accumulate, void* stream);
int tdb_xent_grad(void* logits, int64_t ld, const int64_t* targets, int64_t vocab_start, int valid_cols, int cols,
                  int rows, const float* gstats, float scale, void* stream);

/* ---- optimizer (optim.cu) ----------------------------------------------- */
int tdb_sumsq_partials_count(void);
int tdb_sumsq(const float* g, int64_t n, double* partial, double* out, int accumulate, void* stream);
int tdb_clip_coef(const double* total, float max_norm, double* norm_out, float* coef, const float* loss, int* finite,
                  int* step_counter, void* stream);
int tdb_adamw(float* master, float* grad, float* m, float* v, void* param, int64_t n, int64_t wd_lo0, int64_t wd_hi0,
              int64_t wd_lo1, int64_t wd_hi1, float lr, float beta1, float beta2, float eps, float weight_decay,
              int step, const float* coef, const int* finite, int zero_grad, const int* step_dev, void* stream);
int tdb_to_bf16(const float* src, void* dst, int64_t n, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* TDB_H_ */
