/*
 * CPU oracle for the Qwen3-MoE routing path: integer / ordering work in plain C.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or calls
 * this file: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg use it, and only as the checker.
 *
 * What it restates (reference = charleshong3/nki-moe-7013):
 *   - router logits in fp32 from bf16 activations and bf16 router weight
 *     (qwen.py:260-261 sets the router dtype to fp32), softmax over experts
 *     (qwen.py:263), top-k with the lower expert index winning ties, and the
 *     L1 renormalisation of the chosen affinities (qwen.py:269,
 *     qwen_with_nki.py:2402-2405).  Weights are computed in numpy (oracle.py);
 *     this file only produces the logits and the exact indices.
 *   - the expert-grouped permutation consumed by the blockwise expert kernels
 *     (qwen_with_nki.py:5872-5881): (token, slot) pairs stably grouped by
 *     expert, ascending token id inside an expert.
 *
 * Canonical fp32 reduction order of a router logit (the CUDA kernel computes
 * exactly the same sequence of roundings, so logits and indices are bit-exact):
 *   H is split into groups of 256 elements; inside a group, lane l (0..31)
 *   owns elements [8l, 8l+8).  Lane l accumulates, starting from +0.0f,
 *       for g in 0..H/256-1: for q in 0..7: acc = acc + x[256g+8l+q]*w[...]
 *   The product of two bf16 values is exact in fp32, so `acc + x*w` rounds
 *   once, exactly like the device FMA.  The 32 lane sums are then combined by
 *   a butterfly: for off in 16,8,4,2,1: s[l] = s[l] + s[l ^ off].  The logit
 *   is s[0] (every lane holds the same value since fp32 addition commutes).
 *
 * Build: gcc -O2 -fPIC -shared -ffp-contract=off (oracle/Makefile).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t v) {
    uint32_t u = ((uint32_t)v) << 16;
    float f;
    memcpy(&f, &u, sizeof(f));
    return f;
}

/* logits[t*E + e] = canonical fp32 dot(x[t,:], w[e,:]).  Returns 0, or -1 if
 * H is not a multiple of 256. */
int oracle_router_logits(const uint16_t* x, const uint16_t* w, int64_t T,
                         int64_t H, int64_t E, float* logits) {
    if (H % 256 != 0) return -1;
    const int64_t G = H / 256;
    float* xf = (float*)malloc(sizeof(float) * (size_t)H);
    float* wf = (float*)malloc(sizeof(float) * (size_t)(H * E));
    if (!xf || !wf) { free(xf); free(wf); return -2; }
    for (int64_t i = 0; i < H * E; ++i) wf[i] = bf16_to_f32(w[i]);
    for (int64_t t = 0; t < T; ++t) {
        for (int64_t h = 0; h < H; ++h) xf[h] = bf16_to_f32(x[t * H + h]);
        for (int64_t e = 0; e < E; ++e) {
            const float* we = wf + e * H;
            float s[32];
            for (int l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (int64_t g = 0; g < G; ++g) {
                    const int64_t base = 256 * g + 8 * l;
                    for (int q = 0; q < 8; ++q) {
                        float p = xf[base + q] * we[base + q]; /* exact */
                        acc = acc + p;
                    }
                }
                s[l] = acc;
            }
            for (int off = 16; off >= 1; off >>= 1) {
                float n[32];
                for (int l = 0; l < 32; ++l) n[l] = s[l] + s[l ^ off];
                memcpy(s, n, sizeof(s));
            }
            logits[t * E + e] = s[0];
        }
    }
    free(xf);
    free(wf);
    return 0;
}

/* idx[t*k + j]: the k largest logits of row t in descending order; equal
 * logits are ordered by ascending expert index.  Selection uses the logits,
 * which softmax maps monotonically onto the affinities. */
int oracle_topk(const float* logits, int64_t T, int64_t E, int64_t k,
                int32_t* idx) {
    if (k > E || k <= 0) return -1;
    unsigned char* taken = (unsigned char*)malloc((size_t)E);
    if (!taken) return -2;
    for (int64_t t = 0; t < T; ++t) {
        const float* row = logits + t * E;
        memset(taken, 0, (size_t)E);
        for (int64_t j = 0; j < k; ++j) {
            int64_t best = -1;
            for (int64_t e = 0; e < E; ++e) {
                if (taken[e]) continue;
                if (best < 0 || row[e] > row[best]) best = e; /* strict: lower index kept on ties */
            }
            taken[best] = 1;
            idx[t * k + j] = (int32_t)best;
        }
    }
    free(taken);
    return 0;
}

/* Stable expert-grouped permutation of the T*k (token, slot) pairs.
 *   counts[e]       pairs routed to expert e
 *   offsets[e]      exclusive prefix sum of counts (offsets[E] = T*k)
 *   row_token[r]    token of permuted row r
 *   row_slot[r]     slot j (0..k-1) of permuted row r
 *   slot_row[t*k+j] permuted row of pair (t, j)
 * Inside an expert rows are ordered by ascending token id (each token picks
 * an expert at most once, so this is also pair order). */
int oracle_permute(const int32_t* idx, int64_t T, int64_t E, int64_t k,
                   int32_t* counts, int32_t* offsets, int32_t* row_token,
                   int32_t* row_slot, int32_t* slot_row) {
    int64_t* fill = (int64_t*)calloc((size_t)E, sizeof(int64_t));
    if (!fill) return -2;
    memset(counts, 0, sizeof(int32_t) * (size_t)E);
    for (int64_t p = 0; p < T * k; ++p) {
        int32_t e = idx[p];
        if (e < 0 || e >= E) { free(fill); return -1; }
        counts[e]++;
    }
    offsets[0] = 0;
    for (int64_t e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
    for (int64_t t = 0; t < T; ++t) {
        for (int64_t j = 0; j < k; ++j) {
            int32_t e = idx[t * k + j];
            int64_t r = offsets[e] + fill[e]++;
            row_token[r] = (int32_t)t;
            row_slot[r] = (int32_t)j;
            slot_row[t * k + j] = (int32_t)r;
        }
    }
    free(fill);
    return 0;
}
