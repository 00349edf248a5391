/*
 * pkv_oracle.c -- CPU restatement (fp32) of the reference's decode oracle,
 * TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline, never the engine).
 *
 * Restates cpu_gqa_attention (reference tests/smoke_test.cu:35-74): for each
 * query head, scores s_t = q . k_t / sqrt(d) accumulated in fp32, m = max s,
 * w_t = exp(s_t - m), o = sum w_t v_t / (sum w_t + 1e-8), with KV head
 * qh / G -- here read straight from the paged cache [P, Hkv, page, 128]
 * through the block table, with row-local seq_lens and q/out row indices
 * (the semantics of the reference's paged entry points).  Rows are spread
 * over OpenMP threads.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define D 128

/* IEEE binary16 -> binary32 */
static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do {
                ++e;
                man <<= 1;
            } while ((man & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf16_to_float(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Returns 0, or -1 on an out-of-range page id / length / index. */
int pkv_oracle_paged_decode(const uint16_t* q_source, const uint16_t* k_pages,
                            const uint16_t* v_pages, const int32_t* block_table,
                            const int32_t* seq_lens, const int32_t* q_indices,
                            const int32_t* out_indices, float* out, int B, int q_rows, int out_rows,
                            int Hq, int Hkv, int physical_pages, int page_size, int max_pages,
                            int is_bf16, int n_threads) {
    const int G = Hq / Hkv;
    const float scale = 1.0f / sqrtf((float)D);
    int bad = 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(n_threads) reduction(| : bad)
    for (int task = 0; task < B * Hq; ++task) {
        const int b = task / Hq, qh = task % Hq, kvh = qh / G;
        const int n = seq_lens[b];
        const int qi = q_indices ? q_indices[b] : b;
        const int oi = out_indices ? out_indices[b] : b;
        if (n < 0 || n > max_pages * page_size || qi < 0 || qi >= q_rows || oi < 0 ||
            oi >= out_rows) {
            bad = 1;
            continue;
        }
        float q[D], o[D];
        for (int d = 0; d < D; ++d) {
            const uint16_t raw = q_source[((size_t)qi * Hq + qh) * D + d];
            q[d] = is_bf16 ? bf16_to_float(raw) : half_to_float(raw);
            o[d] = 0.f;
        }
        float* scores = (float*)malloc(sizeof(float) * (n > 0 ? n : 1));
        float m = -3.402823466e38f, l = 0.f;
        for (int t = 0; t < n; ++t) {
            const int page = block_table[(size_t)b * max_pages + t / page_size];
            if (page < 0 || page >= physical_pages) {
                bad = 1;
                scores[t] = -INFINITY;
                continue;
            }
            const uint16_t* k =
                k_pages + (((size_t)page * Hkv + kvh) * page_size + t % page_size) * D;
            float s = 0.f;
            for (int d = 0; d < D; ++d)
                s += q[d] * (is_bf16 ? bf16_to_float(k[d]) : half_to_float(k[d]));
            s *= scale;
            scores[t] = s;
            if (s > m) m = s;
        }
        for (int t = 0; t < n; ++t) {
            const int page = block_table[(size_t)b * max_pages + t / page_size];
            if (page < 0 || page >= physical_pages) continue;
            const uint16_t* v =
                v_pages + (((size_t)page * Hkv + kvh) * page_size + t % page_size) * D;
            const float w = expf(scores[t] - m);
            l += w;
            for (int d = 0; d < D; ++d)
                o[d] += w * (is_bf16 ? bf16_to_float(v[d]) : half_to_float(v[d]));
        }
        for (int d = 0; d < D; ++d) out[((size_t)oi * Hq + qh) * D + d] = o[d] / (l + 1e-8f);
        free(scores);
    }
    return bad ? -1 : 0;
}
