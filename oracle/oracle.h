/*
 * CPU oracle for the paged KV cache + GQA decode-attention path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker used by tests/,
 * __graft_entry__.smoke() and the cpu_baseline leg of bench.py. The product
 * (libtllm_kv.so) never links or calls it.
 *
 * What it restates (reference = AICL-Lab/tiny-llm v2.0.2):
 *   - append: KVCacheManager::appendKV copies num_tokens rows of [Hkv][D]
 *     fp16 at position current_len (src/kv_cache.cpp:206-233); restated here
 *     for a paged pool, with an optional RoPE rotation of K.
 *   - RoPE: rotate-half with freq_i = theta^(-2i/D), angle = pos*freq_i,
 *     out = x*cos + rotate_half(x)*sin (docs/en/architecture/cuda-kernels.md:
 *     291-335; rope_theta in include/tiny_llm/types.h:22). The reference code
 *     has no RoPE kernel, so this part is pinned only by its documented math.
 *   - decode attention: attention_decode_kernel (kernels/attention.cu:11-112):
 *     scores = scale * q.k_t, softmax over t < S, out = sum_t p_t v_t, with
 *     the reference's optional 1/(sum + 1e-6) normalisation (attention.cu:97),
 *     generalised to GQA (kv_head = q_head / G) and per-sequence lengths.
 *
 * fp16 values are carried as uint16_t bit patterns; conversions are IEEE
 * binary16 round-to-nearest-even, written from the format definition.
 * Build with -ffp-contract=off so the RoPE products round exactly as the
 * device code's explicit __fmul_rn/__fadd_rn sequence does.
 */
#ifndef TLLM_ORACLE_H
#define TLLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 <-> binary32 (round to nearest, ties to even). */
uint16_t or_f32_to_f16(float f);
float or_f16_to_f32(uint16_t h);
void or_f32_to_f16_array(const float *src, uint16_t *dst, size_t n);
void or_f16_to_f32_array(const uint16_t *src, float *dst, size_t n);

/* Seeded N(0,1) fp16 generator: splitmix64 stream + Box-Muller in double,
 * rounded to float then to fp16. Same seed -> same bits on every host. */
void or_fill_normal_f16(uint16_t *dst, size_t n, uint64_t seed);

/* RoPE cos/sin tables, [max_pos][D/2] each, fp32:
 * freq_i = pow(theta, -2i/D) (double), angle = pos*freq_i (double),
 * cos/sin evaluated in double and rounded to float. */
void or_rope_table(float *cos_t, float *sin_t, int max_pos, int head_dim, float theta);

/* Rotate one K row of Hkv heads x D at position pos (rotate-half pairs
 * (i, i+D/2)); products and sums each rounded to fp32, result to fp16. */
void or_rope_row(uint16_t *dst, const uint16_t *src, int num_kv_heads, int head_dim,
                 const float *cos_t, const float *sin_t, int pos);

/* Paged pool geometry (matches the product's layout choices). */
typedef struct {
    int num_layers;   /* L */
    int num_kv_heads; /* Hkv */
    int head_dim;     /* D */
    int block_size;   /* bs, tokens per block */
    int num_blocks;   /* NB, blocks per (layer, K|V) region */
    int head_major;   /* 0: block = [bs][Hkv][D]; 1: block = [Hkv][bs][D] */
} or_pool_geom;

/* Element offset of (layer, kv, block, token_in_block, head, d=0) in the
 * pool [L][2][NB][block]; kv 0 = K, 1 = V. */
size_t or_pool_offset(const or_pool_geom *g, int layer, int kv, int block, int tok, int head);

/* Write n tokens (rows [n][Hkv][D]) of one layer at positions pos0..pos0+n-1
 * through block table bt; K rotated by RoPE when cos_t != NULL. */
void or_append(uint16_t *pool, const or_pool_geom *g, const int *bt, int layer, int pos0,
               int n, const uint16_t *k, const uint16_t *v, const float *cos_t,
               const float *sin_t);

/* Gather the first S tokens of one layer back into contiguous [S][Hkv][D]. */
void or_gather(const uint16_t *pool, const or_pool_geom *g, const int *bt, int layer, int S,
               uint16_t *k_out, uint16_t *v_out);

/* Decode attention for one sequence over contiguous K/V [S][Hkv][D]:
 * q [Hq][D] fp16, out [Hq][D] as fp64 math rounded to float.
 * eps is added to the softmax denominator (0, or 1e-6 for the reference
 * kernel's normalisation). S == 0 gives zeros. */
void or_decode_one(const uint16_t *q, const uint16_t *k, const uint16_t *v, int S,
                   int num_q_heads, int num_kv_heads, int head_dim, float scale, double eps,
                   float *out);

/* The timed CPU baseline: fp32 decode over the paged pool, as the reference
 * kernel computes it (fp32 dot products, expf, fp32 sums, 1/(sum+1e-6)),
 * OpenMP over (sequence, kv_head) when threads > 1.
 * q [B][Hq][D] fp16, out [B][Hq][D] fp16, lens[B] attended lengths,
 * bt [B][bt_stride] block tables. Returns the thread count used. */
int or_decode_paged_f32(const uint16_t *pool, const or_pool_geom *g, int layer, int B,
                        const int *bt, int bt_stride, const int *lens, const uint16_t *q,
                        int num_q_heads, float scale, uint16_t *out, int threads);

/* The reference's W8A16 projection (kernels/w8a16_matmul.cu:71-93, the
 * reference kernel; the tiled kernel at :119-218 forms the same sums in the
 * same order): out[r][n] = sum over k ascending of x[r][k] * w_k, where
 * w_k = (float)w[k][n] * scale[k/group][n] rounded to fp32 and each term is
 * fused into the running fp32 sum (nvcc compiles `sum += a * w` to an FMA).
 * x [M][K] fp16, w [K][N] int8 row-major, scales [ceil(K/group)][N] fp16;
 * out [M][N] fp32 (the reference rounds it to fp16). OpenMP over rows and
 * columns when threads > 1. */
void or_w8a16_matmul(const uint16_t *x, const int8_t *w, const uint16_t *scales, int M, int N, int K,
                     int group, float *out, int threads);

#ifdef __cplusplus
}
#endif
#endif
