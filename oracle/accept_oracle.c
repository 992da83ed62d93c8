/*
 * CPU oracle for FlashMap's sampling and acceptance step (test infrastructure:
 * the checker, never the product).
 *
 * Restates the acceptance block of spec_generate in the reference
 * (flashmap/modeling_flashmap.py:553-557 for draft sampling, :579-582 greedy,
 * :583-594 rejection sampling) with the randomness injected from our own
 * Philox4x32-10 stream instead of torch.rand / torch.multinomial, which
 * cannot be reproduced on a GPU.  Every floating-point step below is spelled
 * out in the exact order the CUDA kernels use (flashmap_b200/csrc/ops.cu, philox.cuh),
 * so that GPU and oracle agree bit for bit:
 *
 *   - exp is fm_exp(): Cody-Waite range reduction x = n ln2 + r with ln2 split
 *     into a 16-bit head and a tail, the degree-7 Taylor polynomial of e^r
 *     evaluated by Horner with fused multiply-adds, and an exact power-of-two
 *     scale (two steps below 2^-126 and at 2^128).  Written from the
 *     mathematics; checked against the exact exponential for accuracy in
 *     tests/test_fm_exp_oracle.py.
 *   - row reductions (max, sum of exp) use 256 "threads": thread i walks the
 *     8-element vectors i, i+256, i+512, ... in order; the 256 partials are
 *     combined by the warp tree (offsets 16,8,4,2,1 within each group of 32,
 *     then 4,2,1 over the 8 group results).
 *   - a categorical draw over weights r[0..V) with a uniform u uses 256
 *     contiguous ranges of W = roundup8(ceil(V/256)) elements, their
 *     sequential sums, an inclusive scan (Hillis-Steele in groups of 32, then
 *     a sequential scan of the 8 group totals), target = u * total, and a
 *     two-level search for the first element whose running sum exceeds it.
 *   - the rejection step's bonus draw uses the sliced form of that draw
 *     (fmo_categorical_sliced), so that the GPU spreads it over many blocks:
 *     slices of 256 ranges of 32 elements; per slice the ranges' sequential
 *     sums and the same inclusive scan give the slice total; the slice totals
 *     are summed in order (a sequential prefix), target = u * total picks the
 *     first slice whose prefix exceeds it, and inside that slice the range and
 *     then the element are found as above, each running sum starting from the
 *     prefix of the slices before.
 *   - the rejection step's row sums (fmo_rejection_row_stats) run slice-major
 *     over the same 8192-element slices: in a slice, thread i sums its 4
 *     vectors (slice start + u * 256 + i) in order, the slice total is the
 *     warp tree above, and the slice totals are added in slice order.
 *
 * Philox4x32-10 follows Salmon, Moraes, Dror and Shaw, "Parallel random
 * numbers: as easy as 1, 2, 3" (SC'11): multipliers 0xD2511F53 and
 * 0xCD9E8D57, Weyl key increments 0x9E3779B9 and 0xBB67AE85.
 *
 * Logit rows are float arrays: bf16 logits are widened exactly by the caller.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define NT 256
#define VEC 8
#define CAT_RANGE 32
#define CAT_SLICE (NT * CAT_RANGE)

/* ------------------------------------------------------------------ Philox */

static void philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4])
{
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int round = 0; round < 10; ++round) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        c0 = hi1 ^ c1 ^ k0;
        c1 = lo1;
        c2 = hi0 ^ c3 ^ k1;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

void fmo_philox(const uint32_t ctr[4], uint64_t seed, uint32_t out[4])
{
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    philox4x32_10(ctr, key, out);
}

/* uniform in [0, 1): the top 24 bits of word 0 times 2^-24 */
float fmo_uniform(uint64_t seed, uint32_t a, uint32_t b, uint32_t c, uint32_t purpose)
{
    uint32_t ctr[4] = {a, b, c, purpose}, out[4];
    fmo_philox(ctr, seed, out);
    return (float)(out[0] >> 8) * 5.9604644775390625e-08f; /* 2^-24 */
}

/* ------------------------------------------------------------------ exp */

/* ln2 = LN2_HI + LN2_LO with LN2_HI holding ln2's leading 16 bits, so that
 * n * LN2_HI is exact for |n| < 2^8. */
static const float LN2_HI = 0.693145751953125f;
static const float LN2_LO = 1.42860682030941723212e-6f;
static const float LOG2E = 1.44269502162933349609f;

float fmo_exp(float x)
{
    if (x != x) return x;
    if (x > 88.7228394f) return INFINITY;
    if (x < -103.972084f) return 0.0f;
    float n = rintf(x * LOG2E);
    float r = fmaf(-n, LN2_HI, x);
    r = fmaf(-n, LN2_LO, r);
    /* e^r by Taylor to r^7 (1/k! rounded to float), Horner with fma */
    float p = 1.98412698e-4f;          /* 1/5040 */
    p = fmaf(p, r, 1.38888889e-3f);    /* 1/720 */
    p = fmaf(p, r, 8.33333333e-3f);    /* 1/120 */
    p = fmaf(p, r, 4.16666667e-2f);    /* 1/24 */
    p = fmaf(p, r, 1.66666667e-1f);    /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int e = (int)n;
    union { uint32_t u; float f; } s;
    if (e > 127) { /* e = 128 (x <= 88.7228): 2^127, then 2 (the product stays finite below FLT_MAX) */
        s.u = 254u << 23;
        return (p * s.f) * 2.0f;
    }
    if (e >= -126) {
        s.u = (uint32_t)(e + 127) << 23;
        return p * s.f;
    }
    s.u = (uint32_t)(e + 126 + 127) << 23; /* 2^(e+126), a normal number */
    union { uint32_t u; float f; } t;
    t.u = 1u << 23; /* 2^-126 */
    return (p * s.f) * t.f;
}

/* The formulation of fm_exp that the CUDA kernels evaluate on element pairs
 * (fm_exp2 in flashmap_b200/csrc/philox.cuh), restated for one lane: n by
 * the 1.5 * 2^23 shifter t = x * log2(e) + 1.5 * 2^23 (round half to even,
 * as rintf), the fast path taken when e = bits(t) - 0x4B400000 lies in
 * [-126, 127] (where fmo_exp scales with one multiply), its scale
 * (bits(t) << 23) + bits(1.0f).  *fast tells whether
 * the fast path applies; where it does not, the kernels call fm_exp itself. */
float fmo_exp_shifter(float x, int* fast)
{
    union { float f; uint32_t u; } t, s;
    volatile float y = x * LOG2E; /* rounded before the shifter, as on the GPU */
    t.f = y + 12582912.0f;
    const float n = t.f - 12582912.0f;
    *fast = (uint32_t)(t.u - 0x4B3FFF82u) <= 253u;
    if (!*fast) return fmo_exp(x);
    float r = fmaf(-n, LN2_HI, x);
    r = fmaf(-n, LN2_LO, r);
    float p = 1.98412698e-4f;
    p = fmaf(p, r, 1.38888889e-3f);
    p = fmaf(p, r, 8.33333333e-3f);
    p = fmaf(p, r, 4.16666667e-2f);
    p = fmaf(p, r, 1.66666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    s.u = (t.u << 23) + 0x3F800000u;
    return p * s.f;
}

/* Inputs with bit patterns start, start + stride, ... (count of them, modulo
 * 2^32): how many take the fast path (*fast_count) and how many of those
 * differ from fmo_exp in any bit (the return value). */
int64_t fmo_exp_shifter_sweep(uint32_t start, uint32_t stride, int64_t count, int64_t* fast_count)
{
    int64_t bad = 0, fast_n = 0;
    uint32_t u = start;
    for (int64_t i = 0; i < count; ++i, u += stride) {
        union { uint32_t u; float f; } x, a, b;
        x.u = u;
        int fast = 0;
        a.f = fmo_exp_shifter(x.f, &fast);
        if (!fast) continue;
        ++fast_n;
        b.f = fmo_exp(x.f);
        if (a.u != b.u) ++bad;
    }
    *fast_count = fast_n;
    return bad;
}

/* ------------------------------------------------------------------ reductions */

static float tree_sum(float *part)
{
    float warp_tot[NT / 32];
    for (int w = 0; w < NT / 32; ++w) {
        float *a = part + 32 * w;
        for (int off = 16; off >= 1; off >>= 1)
            for (int l = 0; l < off; ++l) a[l] = a[l] + a[l + off];
        warp_tot[w] = a[0];
    }
    for (int off = NT / 64; off >= 1; off >>= 1)
        for (int l = 0; l < off; ++l) warp_tot[l] = warp_tot[l] + warp_tot[l + off];
    return warp_tot[0];
}

/* max of x_v = logit_v / temperature over a row */
static float row_max(const float *row, int64_t V, float temperature)
{
    float m = -INFINITY;
    for (int64_t v = 0; v < V; ++v) {
        float x = row[v] / temperature;
        if (x > m) m = x;
    }
    return m;
}

/* sum of fm_exp(x_v - m) in the fixed order of the CUDA row kernel */
static float row_sumexp(const float *row, int64_t V, float temperature, float m)
{
    float part[NT];
    int64_t nvec = (V + VEC - 1) / VEC;
    for (int i = 0; i < NT; ++i) {
        float acc = 0.0f;
        for (int64_t vec = i; vec < nvec; vec += NT)
            for (int j = 0; j < VEC; ++j) {
                int64_t v = vec * VEC + j;
                if (v < V) acc = acc + fmo_exp(row[v] / temperature - m);
            }
        part[i] = acc;
    }
    return tree_sum(part);
}

/* The rejection step's sum of fm_exp(x_v - m), in the slice-major order of
 * the CUDA rejection kernels (ops.cu reject_exact_slice): slices of
 * ACC_VPT * NT vectors of VEC; in a slice, thread i sums its ACC_VPT vectors
 * (slice start + u * NT + i, u ascending) element by element, the slice total
 * is the block tree, and the slice totals are added in slice order. */
#define ACC_VPT 4
static float row_sumexp_sliced(const float *row, int64_t V, float temperature, float m)
{
    int64_t nvec = (V + VEC - 1) / VEC;
    int64_t slice_vecs = (int64_t)ACC_VPT * NT;
    float total = 0.0f;
    for (int64_t s0 = 0; s0 < nvec; s0 += slice_vecs) {
        float part[NT];
        for (int i = 0; i < NT; ++i) {
            float acc = 0.0f;
            for (int u = 0; u < ACC_VPT; ++u) {
                int64_t vec = s0 + (int64_t)u * NT + i;
                if (vec >= nvec) break;
                for (int j = 0; j < VEC; ++j) {
                    int64_t v = vec * VEC + j;
                    if (v < V) acc = acc + fmo_exp(row[v] / temperature - m);
                }
            }
            part[i] = acc;
        }
        total = total + tree_sum(part);
    }
    return total;
}

/* (m, S) of a target row in the rejection step (modeling_flashmap.py:583-594) */
void fmo_rejection_row_stats(const float *row, int64_t V, float temperature, float *m_out, float *s_out)
{
    float m = row_max(row, V, temperature);
    *m_out = m;
    *s_out = row_sumexp_sliced(row, V, temperature, m);
}

void fmo_row_stats(const float *row, int64_t V, float temperature, float *m_out, float *s_out)
{
    float m = row_max(row, V, temperature);
    *m_out = m;
    *s_out = row_sumexp(row, V, temperature, m);
}

/* first index of the maximum of a row (torch.argmax semantics) */
int64_t fmo_argmax(const float *row, int64_t V)
{
    int64_t best = 0;
    float bv = row[0];
    for (int64_t v = 1; v < V; ++v) {
        float x = row[v];
        if (x > bv) { bv = x; best = v; }
    }
    return best;
}

/* ------------------------------------------------------------------ categorical draw */

int64_t fmo_range_width(int64_t V)
{
    int64_t w = (V + NT - 1) / NT;
    return (w + VEC - 1) / VEC * VEC;
}

/* inclusive scan of the NT range sums t into h: Hillis-Steele inside each
 * group of 32, then a sequential scan of the group totals added to later groups */
static void block_scan(const float *t, float *h)
{
    for (int w = 0; w < NT / 32; ++w) {
        float *a = h + 32 * w;
        memcpy(a, t + 32 * w, 32 * sizeof(float));
        for (int off = 1; off < 32; off <<= 1) {
            float prev[32];
            memcpy(prev, a, sizeof(prev));
            for (int l = off; l < 32; ++l) a[l] = prev[l - off] + prev[l];
        }
    }
    float base = 0.0f;
    for (int w = 0; w < NT / 32; ++w) {
        float tot = h[32 * w + 31];
        if (w > 0)
            for (int l = 0; l < 32; ++l) h[32 * w + l] = base + h[32 * w + l];
        base = (w == 0) ? tot : base + tot;
    }
}

/* range sums t and their inclusive scan h over slice j of the weights */
static void slice_scan(const float *r, int64_t V, int64_t j, float *t, float *h)
{
    for (int i = 0; i < NT; ++i) {
        float acc = 0.0f;
        int64_t lo = j * CAT_SLICE + (int64_t)i * CAT_RANGE;
        for (int64_t v = lo; v < lo + CAT_RANGE && v < V; ++v) acc = acc + r[v];
        t[i] = acc;
    }
    block_scan(t, h);
}

/* The sliced categorical draw (see the header): the rejection bonus. */
int64_t fmo_categorical_sliced(const float *r, int64_t V, float u)
{
    const int64_t S = (V + CAT_SLICE - 1) / CAT_SLICE;
    float t[NT], h[NT];
    float totals[256], prefix[256];
    if (S > 256) return -1;
    float run = 0.0f;
    for (int64_t j = 0; j < S; ++j) {
        slice_scan(r, V, j, t, h);
        totals[j] = h[NT - 1];
        run = (j == 0) ? totals[j] : run + totals[j];
        prefix[j] = run;
    }
    const float total = prefix[S - 1];
    const float target = u * total;
    int64_t js = -1;
    for (int64_t j = 0; j < S; ++j)
        if (prefix[j] > target) { js = j; break; }
    if (js < 0)
        for (int64_t j = S - 1; j >= 0; --j)
            if (totals[j] > 0.0f) { js = j; break; }
    if (js < 0) return 0; /* all weights zero */
    const float base = js > 0 ? prefix[js - 1] : 0.0f;
    slice_scan(r, V, js, t, h);
    float g[NT];
    for (int i = 0; i < NT; ++i) g[i] = base + h[i];
    int chosen = -1;
    for (int i = 0; i < NT; ++i)
        if (g[i] > target) { chosen = i; break; }
    if (chosen < 0)
        for (int i = NT - 1; i >= 0; --i)
            if (t[i] > 0.0f) { chosen = i; break; }
    if (chosen < 0) return js * CAT_SLICE;
    float acc = chosen > 0 ? g[chosen - 1] : base;
    int64_t lo = js * CAT_SLICE + (int64_t)chosen * CAT_RANGE;
    int64_t hi = lo + CAT_RANGE < V ? lo + CAT_RANGE : V;
    int64_t last_pos = -1;
    for (int64_t v = lo; v < hi; ++v) {
        acc = acc + r[v];
        if (r[v] > 0.0f) last_pos = v;
        if (acc > target) return v;
    }
    return last_pos >= 0 ? last_pos : lo;
}

/* Draw an index from the non-negative weights r[0..V) with uniform u. */
int64_t fmo_categorical(const float *r, int64_t V, float u)
{
    int64_t W = fmo_range_width(V);
    float t[NT], h[NT];
    for (int i = 0; i < NT; ++i) {
        float acc = 0.0f;
        for (int64_t v = (int64_t)i * W; v < (int64_t)(i + 1) * W && v < V; ++v) acc = acc + r[v];
        t[i] = acc;
    }
    block_scan(t, h);
    float total = h[NT - 1];
    float target = u * total;
    int chosen = -1;
    for (int i = 0; i < NT; ++i)
        if (h[i] > target) { chosen = i; break; }
    if (chosen < 0)
        for (int i = NT - 1; i >= 0; --i)
            if (t[i] > 0.0f) { chosen = i; break; }
    if (chosen < 0) return 0; /* all weights zero: never reached for a softmax row */
    float run = chosen > 0 ? h[chosen - 1] : 0.0f;
    int64_t lo = (int64_t)chosen * W, hi = lo + W < V ? lo + W : V;
    int64_t last_pos = -1;
    for (int64_t v = lo; v < hi; ++v) {
        run = run + r[v];
        if (r[v] > 0.0f) last_pos = v;
        if (run > target) return v;
    }
    return last_pos >= 0 ? last_pos : lo;
}

/* ------------------------------------------------------------------ public oracle API */

/* probs[v] = fm_exp(logit_v / T - m) / S for each of `rows` rows */
void fmo_softmax_rows(const float *logits, int64_t rows, int64_t V, float temperature, float *probs)
{
    for (int64_t r = 0; r < rows; ++r) {
        const float *row = logits + r * V;
        float m, s;
        fmo_row_stats(row, V, temperature, &m, &s);
        for (int64_t v = 0; v < V; ++v)
            probs[r * V + v] = fmo_exp(row[v] / temperature - m) / s;
    }
}

/* Draft sampling (:553-557).  temperature <= 0: argmax; else a categorical
 * draw from softmax(logits / T) with uniform (slot, row, offset, purpose 3). */
void fmo_sample_rows(const float *logits, int64_t B, int64_t K, int64_t V, float temperature,
                     uint64_t seed, uint32_t offset, int64_t *tokens, float *probs_out)
{
    for (int64_t b = 0; b < B; ++b)
        for (int64_t k = 0; k < K; ++k) {
            const float *row = logits + (b * K + k) * V;
            if (temperature <= 0.0f) {
                tokens[b * K + k] = fmo_argmax(row, V);
                continue;
            }
            float *p = probs_out + (b * K + k) * V;
            fmo_softmax_rows(row, 1, V, temperature, p);
            float u = fmo_uniform(seed, (uint32_t)k, (uint32_t)b, offset, 3u);
            tokens[b * K + k] = fmo_categorical(p, V, u);
        }
}

/* Greedy acceptance (:579-582) for B rows: target (B, K+1, V), draft (B, K). */
void fmo_accept_greedy(const float *target, const int64_t *draft, int64_t B, int64_t K, int64_t V,
                       int64_t *accepted, int64_t *bonus)
{
    for (int64_t b = 0; b < B; ++b) {
        int64_t acc = 0;
        while (acc < K && draft[b * K + acc] == fmo_argmax(target + (b * (K + 1) + acc) * V, V)) ++acc;
        accepted[b] = acc;
        bonus[b] = fmo_argmax(target + (b * (K + 1) + acc) * V, V);
    }
}

/* Rejection acceptance (:583-594).  target (B, K+1, V) bf16 logits, draft
 * (B, K) tokens, q (B, K, V) fp32 draft probabilities.  u[b,k] uses counter
 * (k, b, offset, 1); the bonus draw (0, b, offset, 2). */
void fmo_accept_rejection(const float *target, const int64_t *draft, const float *q, int64_t B, int64_t K,
                          int64_t V, float temperature, uint64_t seed, uint32_t offset, int64_t *accepted,
                          int64_t *bonus, float *scratch_v)
{
    for (int64_t b = 0; b < B; ++b) {
        int64_t acc = 0;
        for (; acc < K; ++acc) {
            const float *row = target + (b * (K + 1) + acc) * V;
            float m, s;
            fmo_rejection_row_stats(row, V, temperature, &m, &s);
            int64_t d = draft[b * K + acc];
            float p = fmo_exp(row[d] / temperature - m) / s;
            float qd = q[(b * K + acc) * V + d];
            float u = fmo_uniform(seed, (uint32_t)acc, (uint32_t)b, offset, 1u);
            if (!(u * qd < p)) break;
        }
        accepted[b] = acc;
        const float *row = target + (b * (K + 1) + acc) * V;
        float m, s;
        fmo_rejection_row_stats(row, V, temperature, &m, &s);
        int any = 0;
        for (int64_t v = 0; v < V; ++v) {
            float pv = fmo_exp(row[v] / temperature - m) / s;
            if (acc < K) {
                float d = pv - q[(b * K + acc) * V + v];
                pv = d > 0.0f ? d : 0.0f;
            }
            scratch_v[v] = pv;
            if (pv > 0.0f) any = 1;
        }
        if (!any) /* residual.sum() <= 0: fall back to the target distribution */
            for (int64_t v = 0; v < V; ++v) scratch_v[v] = fmo_exp(row[v] / temperature - m) / s;
        float u = fmo_uniform(seed, 0u, (uint32_t)b, offset, 2u);
        bonus[b] = fmo_categorical_sliced(scratch_v, V, u);
    }
}
