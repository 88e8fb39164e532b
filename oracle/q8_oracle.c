/*
 * q8_oracle.c -- CPU restatement of the reference's paged-Q8 attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path: tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs load it; the shipped library never does.
 *
 * Each function restates one step of nick413-bit/gfx906-fa-vllm in plain C:
 *
 *   q8o_quant_block        extension/gfx906_fa_quant.cu:45-85
 *                          (quantize_block_q8_0_halfwarp: fp32 absmax,
 *                           d = amax/127.0f, id = 1.0f/d, rintf, clamp,
 *                           fp16(d) little-endian in bytes 0..1)
 *   q8o_quantize_dense     extension/gfx906_fa_quant.cu:100-129,206-223
 *   q8o_reshape_and_cache  extension/gfx906_fa_quant.cu:150-200,225-253
 *   q8o_gather             extension/gfx906_fa_gather.cu:190-357 (v2 semantics:
 *                          V rows at tok >= seq_len are zero, K rows there are
 *                          left untouched, pages with phys < 0 count as
 *                          fully out of range)
 *   q8o_attention          the fp32 "dequant + softmax" reference the
 *                          attention kernels are held to: K (and V in q8
 *                          mode) dequantised exactly as
 *                          tests/test_q8_roundtrip.py:21-36 does, scores
 *                          scaled by `scale`, the inline-causal rule of
 *                          kernel/fattn-q8.cuh:646-654 (key k is visible to
 *                          query row t iff k <= q_abs_offset + t), the
 *                          additive fp16 mask of kernel/fattn-q8.cuh:628-631,
 *                          the KV_max cut-off of kernel/fattn-q8.cuh:946, and
 *                          softmax + P.V accumulated in double.
 *   q8o_attention_ex       the same with the optional score features:
 *                          the logit soft-cap of kernel/fattn-q8.cuh:638-640
 *                          (softcap * tanh(s / softcap) on the scaled score,
 *                          before the mask); a sliding window and per-head
 *                          sinks as vLLM's attention interface defines them
 *                          (the reference backend rejects both,
 *                          extension/gfx906_fa_backend.py:249-254): key k is
 *                          visible to query position qp iff qp - k < window,
 *                          qp = q_abs + t (or kv_len - n_q + t without
 *                          q_abs), and exp(sink[hq]) joins the softmax
 *                          denominator only.  num_blocks > 0: keys on pages
 *                          whose block-table entry is negative or
 *                          >= num_blocks are dropped.
 *
 * The only fp16 arithmetic needed is float <-> binary16 conversion, written
 * here from the IEEE-754 definition (round to nearest, ties to even).
 *
 * Built with plain gcc (no -ffast-math, so float ops are IEEE single) and
 * OpenMP for the attention loop.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ----------------------------------------------------------------------- */
/* binary16 <-> binary32                                                   */
/* ----------------------------------------------------------------------- */

uint16_t q8o_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {                       /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    }
    int e = (int)exp - 127 + 15;              /* rebias */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);   /* overflow -> inf */
    if (e <= 0) {
        /* subnormal half (or zero): value = man_full * 2^(exp-150);
         * half subnormal unit is 2^-24, so shift = 126 - exp. */
        if (e < -10) return (uint16_t)sign;   /* rounds to zero (below half of 2^-24) */
        uint32_t m = man | 0x800000u;         /* implicit bit */
        int shift = 14 - e;                   /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);          /* carry into exponent is correct */
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;  /* may carry to inf: correct */
    return (uint16_t)(sign | q);
}

float q8o_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {                              /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            man &= 0x3ffu;
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1fu) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline float bf16_to_f32(uint16_t h) {
    uint32_t x = (uint32_t)h << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* dtype codes shared with the CUDA library: 0 = fp16, 1 = bf16, 2 = fp32 */
static inline float load_elem(const void* base, int64_t idx, int dtype) {
    if (dtype == 0) return q8o_f16_to_f32(((const uint16_t*)base)[idx]);
    if (dtype == 1) return bf16_to_f32(((const uint16_t*)base)[idx]);
    return ((const float*)base)[idx];
}

/* ----------------------------------------------------------------------- */
/* Q8_0 block quantiser (gfx906_fa_quant.cu:45-85)                          */
/* ----------------------------------------------------------------------- */

/* float -> int as the GPU converts (the reference kernel's `(int)rintf(q)`
 * on the device): saturating at the int range, NaN -> 0.  C leaves the
 * out-of-range and NaN cases undefined; they occur when a block's absmax is
 * so small that 1/d overflows to infinity (0 * inf = NaN, x * inf = +-inf). */
static inline int device_f2i(float r) {
    if (r != r) return 0;
    if (r >= 2147483647.0f) return 2147483647;
    if (r <= -2147483648.0f) return -2147483647 - 1;
    return (int)r;
}

void q8o_quant_block(const float* v, uint8_t* y) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float d = amax / 127.0f;
    const float id = d > 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = q8o_f32_to_f16(d);
    y[0] = (uint8_t)(dh & 0xffu);
    y[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 32; ++i) {
        float q = v[i] * id;
        int qi = device_f2i(rintf(q));
        if (qi < -128) qi = -128;
        if (qi > 127) qi = 127;
        y[2 + i] = (uint8_t)(int8_t)qi;
    }
}

/* x: [N, D] rows (element type `dtype`), y: [N, D/32*34] bytes. */
void q8o_quantize_dense(const void* x, int dtype, uint8_t* y, int64_t N, int D) {
    const int nb = D / 32;
    for (int64_t r = 0; r < N; ++r) {
        for (int b = 0; b < nb; ++b) {
            float v[32];
            for (int i = 0; i < 32; ++i) v[i] = load_elem(x, r * D + b * 32 + i, dtype);
            q8o_quant_block(v, y + (r * nb + b) * 34);
        }
    }
}

/* key: element strides (tok, head), contiguous D.  cache: byte strides.
 * slot < 0 skips the token (gfx906_fa_quant.cu:168-169). */
void q8o_reshape_and_cache(const void* key, int dtype, const int64_t* slot_mapping,
                           uint8_t* cache, int T, int Hkv, int D, int bs,
                           int64_t key_tok_stride, int64_t key_head_stride,
                           int64_t cache_block_stride, int64_t cache_tok_stride,
                           int64_t cache_head_stride) {
    const int nb = D / 32;
    for (int t = 0; t < T; ++t) {
        int64_t slot = slot_mapping[t];
        if (slot < 0) continue;
        int64_t blk = slot / bs, off = slot % bs;
        for (int h = 0; h < Hkv; ++h) {
            uint8_t* dst = cache + blk * cache_block_stride + off * cache_tok_stride + h * cache_head_stride;
            for (int b = 0; b < nb; ++b) {
                float v[32];
                for (int i = 0; i < 32; ++i)
                    v[i] = load_elem(key, t * key_tok_stride + h * key_head_stride + b * 32 + i, dtype);
                q8o_quant_block(v, dst + b * 34);
            }
        }
    }
}

/* Plain element copy of V into the paged fp16/bf16 cache by slot (what
 * vLLM's reshape_and_cache_flash does for the fp16 V half of the cache). */
void q8o_store_v16(const uint16_t* value, const int64_t* slot_mapping, uint16_t* vcache,
                   int T, int Hkv, int D, int bs, int64_t v_tok_stride, int64_t v_head_stride,
                   int64_t cache_block_stride, int64_t cache_tok_stride, int64_t cache_head_stride) {
    for (int t = 0; t < T; ++t) {
        int64_t slot = slot_mapping[t];
        if (slot < 0) continue;
        int64_t blk = slot / bs, off = slot % bs;
        for (int h = 0; h < Hkv; ++h)
            memcpy(vcache + blk * cache_block_stride + off * cache_tok_stride + h * cache_head_stride,
                   value + t * v_tok_stride + h * v_head_stride, (size_t)D * 2);
    }
}

/* ----------------------------------------------------------------------- */
/* Paged gather (gfx906_fa_gather.cu:190-357)                               */
/* ----------------------------------------------------------------------- */
/* k_cache [NB, bs, Hkv, kbytes] u8, v_cache [NB, bs, Hkv, D] 16-bit,
 * k_out [B, Hkv, Sk, kbytes], v_out [B, Hkv, Sk, D]. */
void q8o_gather(const uint8_t* k_cache, const uint16_t* v_cache, const int32_t* block_table,
                const int32_t* seq_lens, uint8_t* k_out, uint16_t* v_out, int B, int Hkv,
                int Sk, int D, int kbytes, int bs, int max_blocks) {
    for (int s = 0; s < B; ++s) {
        const int L = seq_lens[s];
        for (int h = 0; h < Hkv; ++h) {
            for (int t = 0; t < Sk; ++t) {
                const int pg = t / bs;
                const int phys = pg < max_blocks ? block_table[(int64_t)s * max_blocks + pg] : -1;
                const int page_start = pg * bs;
                const int full_oob = (page_start >= L) || (phys < 0);
                const int valid = !full_oob && t < L;
                uint16_t* vd = v_out + (((int64_t)s * Hkv + h) * Sk + t) * D;
                uint8_t* kd = k_out + (((int64_t)s * Hkv + h) * Sk + t) * kbytes;
                if (valid) {
                    const int64_t row = ((int64_t)phys * bs + (t % bs)) * Hkv + h;
                    memcpy(vd, v_cache + row * D, (size_t)D * 2);
                    memcpy(kd, k_cache + row * kbytes, (size_t)kbytes);
                } else {
                    memset(vd, 0, (size_t)D * 2);
                }
            }
        }
    }
}

/* ----------------------------------------------------------------------- */
/* Dequantisation (tests/test_q8_roundtrip.py:21-36)                        */
/* ----------------------------------------------------------------------- */
void q8o_dequant_row(const uint8_t* row, int D, float* out) {
    for (int b = 0; b < D / 32; ++b) {
        const uint8_t* blk = row + b * 34;
        float d = q8o_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)(int8_t)blk[2 + i] * d;
    }
}

/* Token `t` of a page-transposed Q8_0 V record (this build's own V layout,
 * no reference counterpart): fp16 scale of block j at 2*(j*bs + t), int8 of
 * dim d at 2*(D/32)*bs + d*bs + t.  Same values as q8o_dequant_row of the
 * token's Q8_0 row. */
void q8o_dequant_q8t(const uint8_t* rec, int D, int bs, int t, float* out) {
    const uint8_t* qv = rec + 2 * (D / 32) * bs + t;
    for (int b = 0; b < D / 32; ++b) {
        const uint8_t* s = rec + 2 * (b * bs + t);
        float d = q8o_f16_to_f32((uint16_t)(s[0] | (s[1] << 8)));
        for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)(int8_t)qv[(b * 32 + i) * bs] * d;
    }
}

/* ----------------------------------------------------------------------- */
/* Attention reference                                                     */
/* ----------------------------------------------------------------------- */
/*
 * Generic paged attention over a batch of B sequences.
 *   q        element type q_dtype; row (seq b, token t, head hq) at
 *            q + b*q_seq_stride + (q_start[b] + t)*q_tok_stride + hq*q_head_stride
 *   out      fp32, same addressing with the o_* strides
 *   n_q[b]   query tokens of sequence b, kv_len[b] keys (KV_max)
 *   k_cache  Q8_0 rows, v_cache fp16 rows (v_q8 = 0) or Q8_0 rows (v_q8 = 1);
 *            row of (seq b, key k, kv head h) at
 *            page(b, k/bs)*page_stride + (k%bs)*tok_stride + h*head_stride
 *            (bytes), page(b, p) = block_table[b*max_blocks + p]
 *   causal   q_abs[b] >= 0 : key k visible to token t iff k <= q_abs[b] + t
 *            (q_abs == NULL disables the causal rule)
 *   mask     optional fp16 additive bias, mask[b*mask_seq_stride + t*mask_tok_stride + k]
 * Rows with no visible key are written as zeros.
 */
void q8o_attention_ex(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_tok_stride,
                      int64_t q_head_stride, const int32_t* q_start, const int32_t* n_q,
                      float* out, int64_t o_seq_stride, int64_t o_tok_stride, int64_t o_head_stride,
                      const uint8_t* k_cache, const uint8_t* v_cache, int v_fmt,
                      int64_t k_page_stride, int64_t k_tok_stride, int64_t k_head_stride,
                      int64_t v_page_stride, int64_t v_tok_stride, int64_t v_head_stride,
                      const int32_t* block_table, int max_blocks, int bs, const int32_t* kv_len,
                      const int32_t* q_abs, const uint16_t* mask, int64_t mask_seq_stride,
                      int64_t mask_tok_stride, int B, int Hq, int Hkv, int D, float scale,
                      int nthreads, float softcap, int window, const float* sinks, int num_blocks) {
    const int G = Hq / Hkv;
    /* flatten (b, hq, t) work items */
    int64_t total = 0;
    for (int b = 0; b < B; ++b) total += (int64_t)n_q[b] * Hq;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
#pragma omp parallel
    {
        float qrow[512], krow[512], vrow[512];
        double acc[512];
        int cap = 0;
        double* sc = 0;
#pragma omp for schedule(dynamic, 4)
        for (int64_t item = 0; item < total; ++item) {
            /* decode item -> (b, t, hq) */
            int64_t rem = item;
            int b = 0;
            while (rem >= (int64_t)n_q[b] * Hq) { rem -= (int64_t)n_q[b] * Hq; ++b; }
            const int t = (int)(rem / Hq);
            const int hq = (int)(rem % Hq);
            const int h = hq / G;
            const int L = kv_len[b];
            int kmax = L;                      /* exclusive */
            if (q_abs) {
                int64_t lim = (int64_t)q_abs[b] + t + 1;
                if (lim < kmax) kmax = lim < 0 ? 0 : (int)lim;
            }
            float* o = out + b * o_seq_stride + ((int64_t)q_start[b] + t) * o_tok_stride + hq * o_head_stride;
            if (kmax <= 0) { for (int d = 0; d < D; ++d) o[d] = 0.0f; continue; }
            if (kmax > cap) {
                cap = kmax + 1024;
                sc = (double*)realloc(sc, sizeof(double) * (size_t)cap);
            }
            const int64_t qoff = b * q_seq_stride + ((int64_t)q_start[b] + t) * q_tok_stride + hq * q_head_stride;
            for (int d = 0; d < D; ++d) qrow[d] = load_elem(q, qoff + d, q_dtype);
            double m = -INFINITY;
            int kmin = 0;
            if (window > 0) {
                const int64_t qp = (q_abs ? (int64_t)q_abs[b] : (int64_t)L - n_q[b]) + t;
                const int64_t lo = qp - window + 1;
                kmin = lo < 0 ? 0 : (lo > kmax ? kmax : (int)lo);
            }
            for (int k = 0; k < kmax; ++k) {
                const int phys = block_table[(int64_t)b * max_blocks + k / bs];
                if (k < kmin || (num_blocks > 0 && (phys < 0 || phys >= num_blocks))) {
                    sc[k] = -INFINITY;
                    continue;
                }
                const uint8_t* kr = k_cache + phys * k_page_stride + (k % bs) * k_tok_stride + h * k_head_stride;
                q8o_dequant_row(kr, D, krow);
                double s = 0.0;
                for (int d = 0; d < D; ++d) s += (double)qrow[d] * (double)krow[d];
                s *= (double)scale;
                if (softcap > 0.0f) s = (double)softcap * tanh(s / (double)softcap);
                if (mask) s += (double)q8o_f16_to_f32(mask[b * mask_seq_stride + (int64_t)t * mask_tok_stride + k]);
                sc[k] = s;
                if (s > m) m = s;
            }
            for (int d = 0; d < D; ++d) acc[d] = 0.0;
            double l = 0.0;
            if (m == -INFINITY) { for (int d = 0; d < D; ++d) o[d] = 0.0f; continue; }
            if (sinks) l += exp((double)sinks[hq] - m);
            for (int k = 0; k < kmax; ++k) {
                const double p = exp(sc[k] - m);
                if (p == 0.0) continue;
                l += p;
                const int phys = block_table[(int64_t)b * max_blocks + k / bs];
                const uint8_t* vr = v_cache + phys * v_page_stride + (k % bs) * v_tok_stride + h * v_head_stride;
                if (v_fmt == 3) {
                    q8o_dequant_q8t(v_cache + phys * v_page_stride + h * v_head_stride, D, bs, k % bs, vrow);
                } else if (v_fmt == 2) {
                    q8o_dequant_row(vr, D, vrow);
                } else {
                    const uint16_t* v16 = (const uint16_t*)vr;
                    for (int d = 0; d < D; ++d)
                        vrow[d] = v_fmt == 1 ? bf16_to_f32(v16[d]) : q8o_f16_to_f32(v16[d]);
                }
                for (int d = 0; d < D; ++d) acc[d] += p * (double)vrow[d];
            }
            for (int d = 0; d < D; ++d) o[d] = (float)(acc[d] / l);
        }
        free(sc);
    }
}

void q8o_attention(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_tok_stride,
                   int64_t q_head_stride, const int32_t* q_start, const int32_t* n_q,
                   float* out, int64_t o_seq_stride, int64_t o_tok_stride, int64_t o_head_stride,
                   const uint8_t* k_cache, const uint8_t* v_cache, int v_fmt,
                   int64_t k_page_stride, int64_t k_tok_stride, int64_t k_head_stride,
                   int64_t v_page_stride, int64_t v_tok_stride, int64_t v_head_stride,
                   const int32_t* block_table, int max_blocks, int bs, const int32_t* kv_len,
                   const int32_t* q_abs, const uint16_t* mask, int64_t mask_seq_stride,
                   int64_t mask_tok_stride, int B, int Hq, int Hkv, int D, float scale,
                   int nthreads) {
    q8o_attention_ex(q, q_dtype, q_seq_stride, q_tok_stride, q_head_stride, q_start, n_q, out, o_seq_stride,
                     o_tok_stride, o_head_stride, k_cache, v_cache, v_fmt, k_page_stride, k_tok_stride,
                     k_head_stride, v_page_stride, v_tok_stride, v_head_stride, block_table, max_blocks, bs,
                     kv_len, q_abs, mask, mask_seq_stride, mask_tok_stride, B, Hq, Hkv, D, scale, nthreads,
                     0.0f, 0, 0, 0);
}
