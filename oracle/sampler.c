/*
 * oracle/sampler.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's per-codebook sampling step, used by the
 * tests, by __graft_entry__.smoke() and by bench.py's CPU baseline as the
 * checker.  The product never links or calls this file.
 *
 * What it restates (soraku_inference/model.py):
 *   579-581  CFG merge      merged = u + s * (c - u)          (native formula)
 *   557-559  structural     merged[BOS] = merged[PAD] = -inf
 *   583-584  EOS            merged[EOS] = -inf unless (q == 0 and frame >= min)
 *   694-695  greedy         temperature <= 0 -> argmax (first maximal index)
 *   696      temperature    filtered = merged / temperature   (IEEE division,
 *                           then + 0.0f, which folds -0 into +0)
 *   697-699  top-k          cutoff = k-th largest (duplicates counted);
 *                           entries < cutoff removed, ties at the cutoff kept
 *   700-706  top-p          sort descending, cum = cumsum(softmax(sorted)),
 *                           remove[i] = cum[i-1] > p, remove[0] = False
 *   707-708  draw           softmax over the kept set, one multinomial draw
 *
 * torch.multinomial cannot be reproduced, so the draw is restated with an
 * explicit uniform u in [0, 1): the kept candidates are ordered by (value
 * descending, index ascending); e_j = exp(f_j - f_0) with the exp below; the
 * top-p cumulative is the sequential FP32 sum of e_j / S1 (S1 = sequential sum
 * of every candidate's e_j); the draw is the first kept j whose sequential FP32
 * running sum of e_j exceeds u * S2 (S2 = sequential sum over the kept set),
 * or the last kept j with e_j > 0 when rounding leaves none.  The CUDA kernel
 * in soraku_tts_b200/csrc/sampler.cuh performs the same IEEE operations in the
 * same order, so both return the same code for the same logits and uniform.
 *
 * Built with -ffp-contract=off: every multiply and add rounds separately
 * except where fmaf() asks for a fused operation.
 *
 * exp: Cody & Waite range reduction (W. J. Cody, W. Waite, "Software Manual
 * for the Elementary Functions", 1980): n = rint(x / ln2), r = x - n*ln2 with
 * ln2 split into a 16-bit head and a tail, then the degree-7 Taylor polynomial
 * of e^r in Horner form with FMA, scaled by 2^n.  Results below 2^-126 are
 * flushed to zero.
 *
 * Philox4x32-10: J. K. Salmon, M. A. Moraes, R. O. Dror, D. E. Shaw,
 * "Parallel random numbers: as easy as 1, 2, 3", SC'11.  Counter =
 * (q, frame, request, 0), key = (seed low 32 bits, seed high 32 bits);
 * u = (word0 >> 8) * 2^-24.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ exp */
static const float ORC_LOG2E = 1.44269502162933349609375f;   /* fl(1/ln 2) */
static const float ORC_LN2_HI = 0.693145751953125f;          /* 16-bit head */
static const float ORC_LN2_LO = 1.428606765330187045e-06f;   /* ln2 - head */

float orc_exp(float x) {
    if (x != x) return x;
    if (x == -INFINITY) return 0.0f;
    if (x < -104.0f) return 0.0f;
    if (x > 88.7f) return INFINITY;
    float t = x * ORC_LOG2E;
    float n = rintf(t);
    float r = fmaf(-n, ORC_LN2_HI, x);
    r = fmaf(-n, ORC_LN2_LO, r);
    float p = 1.984126984126984e-04f;          /* 1/7! */
    p = fmaf(p, r, 1.388888888888889e-03f);    /* 1/6! */
    p = fmaf(p, r, 8.333333333333333e-03f);    /* 1/5! */
    p = fmaf(p, r, 4.166666666666667e-02f);    /* 1/4! */
    p = fmaf(p, r, 1.666666666666667e-01f);    /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni < -126) return 0.0f;
    if (ni > 127) return INFINITY;
    uint32_t bits = (uint32_t)(ni + 127) << 23;
    float scale;
    memcpy(&scale, &bits, sizeof scale);
    float y = p * scale;
    /* flush a subnormal product the same way the device code does */
    if (y < 1.17549435e-38f) return 0.0f;
    return y;
}

/* --------------------------------------------------------------- philox */
static void mulhilo32(uint32_t a, uint32_t b, uint32_t *hi, uint32_t *lo) {
    uint64_t p = (uint64_t)a * (uint64_t)b;
    *hi = (uint32_t)(p >> 32);
    *lo = (uint32_t)p;
}

void orc_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int round = 0; round < 10; ++round) {
        if (round > 0) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        uint32_t hi0, lo0, hi1, lo1;
        mulhilo32(0xD2511F53u, c0, &hi0, &lo0);
        mulhilo32(0xCD9E8D57u, c2, &hi1, &lo1);
        uint32_t n0 = hi1 ^ c1 ^ k0;
        uint32_t n1 = lo1;
        uint32_t n2 = hi0 ^ c3 ^ k1;
        uint32_t n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

float orc_uniform(uint64_t seed, uint32_t request, uint32_t frame, uint32_t q) {
    uint32_t ctr[4] = {q, frame, request, 0u};
    uint32_t key[2] = {(uint32_t)(seed & 0xffffffffu), (uint32_t)(seed >> 32)};
    uint32_t out[4];
    orc_philox4x32_10(ctr, key, out);
    return (float)(out[0] >> 8) * (1.0f / 16777216.0f);
}

/* -------------------------------------------------------------- sampler */
typedef struct {
    float v;
    int i;
} orc_cand;

static int cmp_cand(const void *a, const void *b) {
    const orc_cand *x = (const orc_cand *)a, *y = (const orc_cand *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

static int cmp_desc(const void *a, const void *b) {
    float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

/*
 * Returns the drawn code.  uncond may be NULL (no CFG).  top_k <= 0 or >= V
 * disables top-k; top_p outside (0, 1) disables top-p.  merged_out (length V,
 * optional) receives the masked merged logits before temperature; info
 * (optional, 4 ints) receives {n_candidates, n_kept, pick_rank, greedy}.
 */
int orc_sample(const float *cond, const float *uncond, int V, float cfg,
               float temperature, int top_k, float top_p, int mask_eos,
               int bos, int pad, int eos, float u, float *merged_out, int *info) {
    float *m = (float *)malloc(sizeof(float) * (size_t)V);
    for (int i = 0; i < V; ++i) {
        float c = cond[i];
        if (uncond) {
            float un = uncond[i];
            float diff = c - un;
            float scaled = cfg * diff;
            m[i] = un + scaled;
        } else {
            m[i] = c;
        }
    }
    if (bos >= 0 && bos < V) m[bos] = -INFINITY;
    if (pad >= 0 && pad < V) m[pad] = -INFINITY;
    if (mask_eos && eos >= 0 && eos < V) m[eos] = -INFINITY;
    if (merged_out) memcpy(merged_out, m, sizeof(float) * (size_t)V);

    int code;
    if (!(temperature > 0.0f)) {
        int best = 0;
        for (int i = 1; i < V; ++i)
            if (m[i] > m[best]) best = i;
        if (info) { info[0] = V; info[1] = 1; info[2] = 0; info[3] = 1; }
        free(m);
        return best;
    }
    /* the trailing + 0.0f folds -0 into +0 so that ordering by value is total */
    for (int i = 0; i < V; ++i) m[i] = m[i] / temperature + 0.0f;

    int topk_on = top_k > 0 && top_k < V;
    float cutoff = -INFINITY;
    if (topk_on) {
        float *tmp = (float *)malloc(sizeof(float) * (size_t)V);
        memcpy(tmp, m, sizeof(float) * (size_t)V);
        qsort(tmp, (size_t)V, sizeof(float), cmp_desc);
        cutoff = tmp[top_k - 1];
        free(tmp);
    }
    orc_cand *cand = (orc_cand *)malloc(sizeof(orc_cand) * (size_t)V);
    int n = 0;
    for (int i = 0; i < V; ++i) {
        if (!topk_on || !(m[i] < cutoff)) {
            cand[n].v = m[i];
            cand[n].i = i;
            ++n;
        }
    }
    qsort(cand, (size_t)n, sizeof(orc_cand), cmp_cand);
    float top = cand[0].v;
    float *e = (float *)malloc(sizeof(float) * (size_t)n);
    for (int j = 0; j < n; ++j) e[j] = orc_exp(cand[j].v - top);

    int keep = n;
    if (top_p > 0.0f && top_p < 1.0f) {
        float s1 = 0.0f;
        for (int j = 0; j < n; ++j) s1 = s1 + e[j];
        float cum = 0.0f;
        for (int j = 0; j < n; ++j) {
            cum = cum + e[j] / s1;
            if (cum > top_p) {
                keep = j + 1;
                break;
            }
        }
    }
    float s2 = 0.0f;
    for (int j = 0; j < keep; ++j) s2 = s2 + e[j];
    float t = u * s2;
    int pick = -1;
    float run = 0.0f;
    for (int j = 0; j < keep; ++j) {
        run = run + e[j];
        if (run > t) {
            pick = j;
            break;
        }
    }
    if (pick < 0) {
        pick = 0;
        for (int j = keep - 1; j >= 0; --j)
            if (e[j] > 0.0f) { pick = j; break; }
    }
    code = cand[pick].i;
    if (info) { info[0] = n; info[1] = keep; info[2] = pick; info[3] = 0; }
    free(e);
    free(cand);
    free(m);
    return code;
}
