/*
 * asa_oracle.c -- CPU restatement of the reference's α-entmax block-sparse
 * attention arithmetic (mvideet/Adaptive-Splash-Attention,
 * source/adasplashattention.cu).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the parity tests,
 * the smoke check and bench.py's CPU-baseline leg compare the CUDA engine
 * against.  Nothing in the product (the splash_attention package, the C-ABI
 * library, the CUDA kernels) links, imports or calls it.
 *
 * Every function names the reference lines it follows.  Floating-point
 * details mirror what nvcc emits for the reference by default (-fmad=true):
 * every `acc += a*b` dot-product step is an explicit fmaf, `(α-1)*s - τ` is
 * fmaf(α-1, s, -τ); this file is compiled with -ffp-contract=off so the host
 * compiler adds no contractions of its own.  powf is libm's powf, which is
 * correctly rounded for the integer exponents the configured α values
 * produce.
 *
 * Pinning: the golden fixtures under tests/golden/ were produced by running
 * the reference's own CUDA kernels (built from the reference source by
 * oracle/build_ref.py) on a B200; tests/test_oracle_golden.py checks this
 * file against them.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <stddef.h>

#define ASA_EPS 1e-8f          /* adasplashattention.cu:21 */
#define ASA_MAX_HALLEY 5       /* adasplashattention.cu:22 */
#define ASA_KMAX 64

typedef struct {
    int BH;          /* B*H rows, each an independent head            */
    int NQ, NK, d;   /* query rows, key rows, head dim                */
    int BM, BN;      /* query-block and key-block sizes (mask tiles)  */
    int k_keep;      /* K_KEEP: top-k kept per query                  */
    float alpha;     /* entmax alpha (clamped to [1.05, 3] inside)    */
    float sm_scale;  /* score scale                                   */
    int causal;      /* 0 => every key visible (reference: Q_idx = INT32_MAX) */
    int ref_tile_load; /* 1 => reproduce the reference's tile-load zeroing (below) */
} asa_oracle_cfg;

static float clamp_alpha(float a) {            /* adasplashattention.cu:52, :547 */
    return fmaxf(1.05f, fminf(a, 3.0f));
}

static int visible(const asa_oracle_cfg* c, int qpos, int kpos) {
    /* adasplashattention.cu:181,189,291,299: key visible iff K_idx <= Q_idx */
    return c->causal ? (kpos <= qpos) : 1;
}

/* Dot product in the reference's order: t ascending, one FMA per step
 * (adasplashattention.cu:190-193, 301-305, 411-414). */
static float dot_chain(const float* a, const float* b, int d) {
    float s = 0.0f;
    for (int t = 0; t < d; ++t) s = fmaf(a[t], b[t], s);
    return s;
}

static float score(const asa_oracle_cfg* c, const float* q, const float* k) {
    float s = dot_chain(q, k, c->d);
    s *= c->sm_scale;                          /* :195 */
    s = fmaxf(s, -10.0f);                      /* :196 */
    s = fminf(s, 10.0f);                       /* :197 */
    return s;
}

/* The reference stages each K (and V) tile in shared memory with one
 * thread per query of the query block, and each loading thread zeroes the
 * elements of keys that ITS OWN query cannot see:
 *   Ktile[x] = (K_idx[kn] <= seq_q_of_loader) ? K[kn][dim] : 0
 * with x = col*d + dim, loader thread x % BLOCK_M, i.e. loader query
 * qb*BLOCK_M + (x % BLOCK_M)  (adasplashattention.cu:176-183, 285-294,
 * 398-406, 442-450).  Consumers then skip only the keys invisible to
 * themselves (:187-189), so a visible key's row may be read with some
 * elements zeroed.  This reproduces that: row_of() returns key kn's row as
 * the consumers of query block qb see it.  A loader query >= NQ belongs to
 * a thread that exited before loading (:156-158, :258, :368); the
 * reference then reads stale shared memory, which cannot be reproduced, and
 * here such an element is taken as loaded. */
static const float* row_of(const asa_oracle_cfg* c, const float* src, int bh, int qb, int kn,
                           const int32_t* Qidx, const int32_t* Kidx, float* buf) {
    const float* r = src + ((size_t)bh * c->NK + kn) * c->d;
    if (!c->ref_tile_load || !c->causal) return r;
    const int col = kn % c->BN;
    const int kpos = Kidx[(size_t)bh * c->NK + kn];
    for (int t = 0; t < c->d; ++t) {
        const int lq = qb * c->BM + (int)(((long long)col * c->d + t) % c->BM);
        const int keep = lq >= c->NQ || kpos <= Qidx[(size_t)bh * c->NQ + lq];
        buf[t] = keep ? r[t] : 0.0f;
    }
    return buf;
}

/* adasplashattention.cu:35-49: descending list, strict '>' so the earlier
 * key keeps its place on ties; a value that does not beat the last entry is
 * dropped. */
static void insert_topk(float val, int idx, float* vals, int* inds, int k) {
    int j = k - 1;
    while (j >= 0 && val > vals[j]) {
        if (j < k - 1) { vals[j + 1] = vals[j]; inds[j + 1] = inds[j]; }
        --j;
    }
    ++j;
    if (j < k) { vals[j] = val; inds[j] = idx; }
}

/* adasplashattention.cu:51-148 (entmax_threshold with full=true): at most
 * five Halley steps on f(τ) = Σ_j relu((α-1)s_j - τ)^{1/(α-1)} - 1 with a
 * bisection safeguard.  The second-derivative coefficient inv·(inv+1-α) is
 * the reference's (:85).  Only τ is returned; the normalised p buffer the
 * reference also fills is discarded by its caller (:205-207). */
float asa_oracle_entmax_tau(const float* s, int k, float alpha_in) {
    const float alpha = clamp_alpha(alpha_in);
    const float am1 = alpha - 1.0f;
    const float inv = 1.0f / am1;
    const float e2 = (2.0f - alpha) * inv;
    const float e3 = (3.0f - 2.0f * alpha) * inv;
    const float c2 = inv * (inv + 1.0f - alpha);
    const float s_max = s[0], s_min = s[k - 1];
    float lo = fmaf(am1, s_min, -2.0f);
    float hi = fmaf(am1, s_max, 2.0f);
    float tau = 0.5f * (lo + hi);
    for (int it = 0; it < ASA_MAX_HALLEY; ++it) {
        float f = -1.0f, fp = 0.0f, fpp = 0.0f;
        for (int j = 0; j < k; ++j) {
            float u = fmaf(am1, s[j], -tau);
            if (u <= 0.0f) break;
            float uc = fmaxf(u, ASA_EPS);
            float up = powf(uc, inv);
            if (isnan(up) || isinf(up)) up = 0.0f;
            f += up;
            float dt = -inv * powf(uc, e2);
            if (isfinite(dt)) fp += dt;
            float st = c2 * powf(uc, e3);
            if (isfinite(st)) fpp += st;
        }
        if (fabsf(f) < 1e-4f) break;
        float tn = tau;
        if (fabsf(fp) > ASA_EPS) {
            float denom = fmaf(2.0f * fp, fp, -(f * fpp));
            if (fabsf(denom) > ASA_EPS) tn = tau - 2.0f * f * fp / denom;
        }
        if (!(tn >= lo && tn <= hi)) tn = 0.5f * (lo + hi);
        f = -1.0f;
        for (int j = 0; j < k; ++j) {
            float u = fmaf(am1, s[j], -tn);
            if (u <= 0.0f) break;
            float up = powf(fmaxf(u, ASA_EPS), inv);
            if (isfinite(up)) f += up;
        }
        if (f > 0.0f) lo = tn; else hi = tn;
        tau = tn;
        tau = fmaxf(tau, fmaf(s_min, am1, -10.0f));
        tau = fminf(tau, fmaf(s_max, am1, 10.0f));
    }
    return tau;
}

/* adasplashattention.cu:150-217 (build_mask_kernel): per query, a causal
 * scan of every key in ascending order, top-k of the clamped scores, τ from
 * the top-k, and M[bh, q/BM, key/BN] = 1 for every kept key.
 * M must hold BH*nQB*nKB bytes; it is zeroed here.  topv/topi (optional,
 * BH*NQ*k_keep each) receive the final top-k lists. */
void asa_oracle_tau_mask(const asa_oracle_cfg* c, const float* Q, const float* K,
                         const int32_t* Qidx, const int32_t* Kidx,
                         float* tau, uint8_t* M, float* topv, int32_t* topi) {
    const int nQB = (c->NQ + c->BM - 1) / c->BM;
    const int nKB = (c->NK + c->BN - 1) / c->BN;
    const int k = c->k_keep;
    memset(M, 0, (size_t)c->BH * nQB * nKB);
    const float alpha = clamp_alpha(c->alpha);
    #pragma omp parallel for schedule(dynamic, 16) collapse(2)
    for (int bh = 0; bh < c->BH; ++bh) {
        for (int q = 0; q < c->NQ; ++q) {
            float vals[ASA_KMAX]; int inds[ASA_KMAX];
            float kbuf[512];
            for (int i = 0; i < k; ++i) { vals[i] = -1e6f; inds[i] = -1; }   /* :166-172 */
            const size_t qi = (size_t)bh * c->NQ + q;
            const float* qrow = Q + qi * c->d;
            const int qpos = Qidx[qi];
            for (int kn = 0; kn < c->NK; ++kn) {
                if (!visible(c, qpos, Kidx[(size_t)bh * c->NK + kn])) continue;
                float s = score(c, qrow, row_of(c, K, bh, q / c->BM, kn, Qidx, Kidx, kbuf));
                insert_topk(s, kn, vals, inds, k);
            }
            tau[qi] = asa_oracle_entmax_tau(vals, k, alpha);
            const size_t base = ((size_t)bh * nQB + q / c->BM) * nKB;
            for (int i = 0; i < k; ++i) {
                if (inds[i] < 0) continue;
                M[base + inds[i] / c->BN] = 1;   /* benign same-value race, as :215 */
            }
            if (topv) for (int i = 0; i < k; ++i) topv[qi * k + i] = vals[i];
            if (topi) for (int i = 0; i < k; ++i) topi[qi * k + i] = inds[i];
        }
    }
}

/* adasplashattention.cu:219-242 (build_lookup_kernel): CSR of M.
 * ptr: BH*(nQB+1), idx: BH*nQB*nKB (zero padded). */
void asa_oracle_csr(const asa_oracle_cfg* c, const uint8_t* M, int32_t* ptr, int32_t* idx) {
    const int nQB = (c->NQ + c->BM - 1) / c->BM;
    const int nKB = (c->NK + c->BN - 1) / c->BN;
    for (int bh = 0; bh < c->BH; ++bh) {
        const uint8_t* m = M + (size_t)bh * nQB * nKB;
        int32_t* p = ptr + (size_t)bh * (nQB + 1);
        int32_t* ix = idx + (size_t)bh * nQB * nKB;
        memset(ix, 0, sizeof(int32_t) * (size_t)nQB * nKB);
        p[0] = 0;
        for (int i = 0; i < nQB; ++i) {
            int cnt = 0;
            for (int j = 0; j < nKB; ++j) cnt += m[i * nKB + j];
            p[i + 1] = p[i] + cnt;
        }
        for (int i = 0; i < nQB; ++i) {
            int w = p[i];
            for (int j = 0; j < nKB; ++j) if (m[i * nKB + j]) ix[w++] = j;
        }
    }
}

static float entmax_p(float u, float inv) {
    /* adasplashattention.cu:311-316 */
    float p = (u > 0.0f) ? powf(fmaxf(u, ASA_EPS), inv) : 0.0f;
    if (isnan(p) || isinf(p)) p = 0.0f;
    return p;
}

/* Walk every visible key of every active tile of query (bh,q) in the
 * reference's order (CSR order, then key ascending) and accumulate the
 * un-normalised numerator acc and the normaliser n
 * (adasplashattention.cu:282-326 and :395-434). */
static float row_accumulate(const asa_oracle_cfg* c, int bh, int q,
                            const float* Q, const float* K, const float* V,
                            const int32_t* Qidx, const int32_t* Kidx, float tq,
                            const int32_t* ptr, const int32_t* idx, float* acc) {
    const int nQB = (c->NQ + c->BM - 1) / c->BM;
    const int nKB = (c->NK + c->BN - 1) / c->BN;
    const float alpha = clamp_alpha(c->alpha);
    const float am1 = alpha - 1.0f, inv = 1.0f / am1;
    const size_t qi = (size_t)bh * c->NQ + q;
    const float* qrow = Q + qi * c->d;
    const int qpos = Qidx[qi];
    const int32_t* p = ptr + (size_t)bh * (nQB + 1);
    const int32_t* ix = idx + (size_t)bh * nQB * nKB;
    const int qb = q / c->BM;
    float n = 0.0f;
    for (int t = 0; t < c->d; ++t) acc[t] = 0.0f;
    for (int e = p[qb]; e < p[qb + 1]; ++e) {
        const int start = ix[e] * c->BN;
        for (int j = 0; j < c->BN; ++j) {
            const int kn = start + j;
            if (kn >= c->NK) break;
            const size_t ki = (size_t)bh * c->NK + kn;
            if (!visible(c, qpos, Kidx[ki])) continue;
            float kbuf[512], vbuf[512];
            float s = score(c, qrow, row_of(c, K, bh, qb, kn, Qidx, Kidx, kbuf));
            float u = fmaf(am1, s, -tq);
            float pr = entmax_p(u, inv);
            n += pr;
            const float* v = row_of(c, V, bh, qb, kn, Qidx, Kidx, vbuf);
            for (int t = 0; t < c->d; ++t) acc[t] = fmaf(pr, v[t], acc[t]);
        }
    }
    return n;
}

/* adasplashattention.cu:244-341 (splash_forward_sparse): O = acc/(n+EPS),
 * non-finite -> 0.  rownorm (optional) receives n. */
void asa_oracle_forward(const asa_oracle_cfg* c, const float* Q, const float* K, const float* V,
                        const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                        const int32_t* ptr, const int32_t* idx, float* O, float* rownorm) {
    #pragma omp parallel
    {
        float* acc = (float*)malloc(sizeof(float) * c->d);
        #pragma omp for schedule(dynamic, 16) collapse(2)
        for (int bh = 0; bh < c->BH; ++bh) {
            for (int q = 0; q < c->NQ; ++q) {
                const size_t qi = (size_t)bh * c->NQ + q;
                float n = row_accumulate(c, bh, q, Q, K, V, Qidx, Kidx, tau[qi], ptr, idx, acc);
                float invN = 1.0f / (n + ASA_EPS);
                for (int t = 0; t < c->d; ++t) {
                    float o = acc[t] * invN;
                    if (isnan(o) || isinf(o)) o = 0.0f;
                    O[qi * c->d + t] = o;
                }
                if (rownorm) rownorm[qi] = n;
            }
        }
        free(acc);
    }
}

/* Pair gradient of the fixed-τ objective for (q, k), adasplashattention.cu:
 * 463-507.  Returns p through *p_out and grad_s. */
static float pair_grad(const asa_oracle_cfg* c, const float* qrow, const float* krow,
                       const float* vrow, const float* dorow, float tq, float invN,
                       float accdO, float* p_out) {
    const float alpha = clamp_alpha(c->alpha);
    const float am1 = alpha - 1.0f, inv = 1.0f / am1;
    const float e2 = (2.0f - alpha) / (alpha - 1.0f);           /* :495 */
    float s = score(c, qrow, krow);
    float u = fmaf(am1, s, -tq);
    float p = entmax_p(u, inv);
    float dp = 0.0f;
    for (int t = 0; t < c->d; ++t) dp = fmaf(vrow[t] * dorow[t], invN, dp);   /* :481-485 */
    dp = fmaf(accdO, -invN * invN, dp);                                        /* :491 */
    float gu = 0.0f;
    if (u > ASA_EPS && fabsf(alpha - 1.0f) > ASA_EPS) {
        float pw = powf(fmaxf(u, ASA_EPS), e2);
        if (isfinite(pw)) gu = (1.0f / (alpha - 1.0f)) * pw * dp;
    }
    float gs = gu * (alpha - 1.0f);
    if (!isfinite(gs)) gs = 0.0f;
    *p_out = p;
    return gs;
}

/* adasplashattention.cu:343-535 (splash_backward_sparse): the fixed-τ
 * gradient.  Per visible pair (q,k) of an active tile:
 *   pb = p/n;  dV_k += pb·dO_q
 *   dp = Σ_t v_t·dO_t·invN + (acc·dO)·(-invN²)
 *   g  = (1/(α-1))·u^{(2-α)/(α-1)}·dp·(α-1)   if u > EPS (else 0)
 *   dQ_q += g·k·sm_scale;  dK_k += g·q·sm_scale
 * The reference accumulates dK/dV with fp32 atomics in arbitrary order; this
 * restatement computes dQ per query row and dK/dV per key row (both loops
 * over the same pairs), which is deterministic.  The host-side scrub
 * (:684-697) is applied by the caller (oracle.py host_scrub). */
void asa_oracle_backward(const asa_oracle_cfg* c, const float* Q, const float* K, const float* V,
                         const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                         const int32_t* ptr, const int32_t* idx, const float* dO,
                         float* dQ, float* dK, float* dV) {
    const int nQB = (c->NQ + c->BM - 1) / c->BM;
    const int nKB = (c->NK + c->BN - 1) / c->BN;
    const int d = c->d;
    const size_t rows = (size_t)c->BH * c->NQ;
    float* invN = (float*)malloc(sizeof(float) * rows);
    float* accdO = (float*)malloc(sizeof(float) * rows);
    uint8_t* active = (uint8_t*)calloc((size_t)c->BH * nQB * nKB, 1);
    for (int bh = 0; bh < c->BH; ++bh) {
        const int32_t* p = ptr + (size_t)bh * (nQB + 1);
        const int32_t* ix = idx + (size_t)bh * nQB * nKB;
        for (int qb = 0; qb < nQB; ++qb)
            for (int e = p[qb]; e < p[qb + 1]; ++e)
                active[((size_t)bh * nQB + qb) * nKB + ix[e]] = 1;
    }
    /* pass 1 (:395-437): per-row n and acc·dO */
    #pragma omp parallel
    {
        float* acc = (float*)malloc(sizeof(float) * d);
        #pragma omp for schedule(dynamic, 16) collapse(2)
        for (int bh = 0; bh < c->BH; ++bh)
            for (int q = 0; q < c->NQ; ++q) {
                const size_t qi = (size_t)bh * c->NQ + q;
                float n = row_accumulate(c, bh, q, Q, K, V, Qidx, Kidx, tau[qi], ptr, idx, acc);
                invN[qi] = 1.0f / (n + ASA_EPS);
                accdO[qi] = dot_chain(acc, dO + qi * d, d);    /* :487-490 */
            }
        free(acc);
    }
    /* dQ per query row (:509-514, :524-534) */
    #pragma omp parallel for schedule(dynamic, 16) collapse(2)
    for (int bh = 0; bh < c->BH; ++bh)
        for (int q = 0; q < c->NQ; ++q) {
            const size_t qi = (size_t)bh * c->NQ + q;
            const int qpos = Qidx[qi];
            float* dq = dQ + qi * d;
            for (int t = 0; t < d; ++t) dq[t] = 0.0f;
            const int32_t* p = ptr + (size_t)bh * (nQB + 1);
            const int32_t* ix = idx + (size_t)bh * nQB * nKB;
            const int qb = q / c->BM;
            for (int e = p[qb]; e < p[qb + 1]; ++e) {
                const int start = ix[e] * c->BN;
                for (int j = 0; j < c->BN; ++j) {
                    const int kn = start + j;
                    if (kn >= c->NK) break;
                    const size_t ki = (size_t)bh * c->NK + kn;
                    if (!visible(c, qpos, Kidx[ki])) continue;
                    float pr, kbuf[512], vbuf[512];
                    const float* kr = row_of(c, K, bh, qb, kn, Qidx, Kidx, kbuf);
                    const float* vr = row_of(c, V, bh, qb, kn, Qidx, Kidx, vbuf);
                    float gs = pair_grad(c, Q + qi * d, kr, vr, dO + qi * d,
                                         tau[qi], invN[qi], accdO[qi], &pr);
                    for (int t = 0; t < d; ++t) {
                        float v = gs * kr[t] * c->sm_scale;
                        if (isfinite(v)) dq[t] += v;
                    }
                }
            }
            for (int t = 0; t < d; ++t) if (!isfinite(dq[t])) dq[t] = 0.0f;
        }
    /* dK, dV per key row (:471-479, :516-519) */
    #pragma omp parallel for schedule(dynamic, 16) collapse(2)
    for (int bh = 0; bh < c->BH; ++bh)
        for (int kn = 0; kn < c->NK; ++kn) {
            const size_t ki = (size_t)bh * c->NK + kn;
            float* dk = dK + ki * d;
            float* dv = dV + ki * d;
            for (int t = 0; t < d; ++t) { dk[t] = 0.0f; dv[t] = 0.0f; }
            const int kb = kn / c->BN;
            const int kpos = Kidx[ki];
            for (int q = 0; q < c->NQ; ++q) {
                const size_t qi = (size_t)bh * c->NQ + q;
                if (!active[((size_t)bh * nQB + q / c->BM) * nKB + kb]) continue;
                if (!visible(c, Qidx[qi], kpos)) continue;
                float pr, kbuf[512], vbuf[512];
                const float* kr = row_of(c, K, bh, q / c->BM, kn, Qidx, Kidx, kbuf);
                const float* vr = row_of(c, V, bh, q / c->BM, kn, Qidx, Kidx, vbuf);
                float gs = pair_grad(c, Q + qi * d, kr, vr, dO + qi * d,
                                     tau[qi], invN[qi], accdO[qi], &pr);
                const float pb = pr * invN[qi];
                const float* g = dO + qi * d;
                const float* qr = Q + qi * d;
                for (int t = 0; t < d; ++t) {
                    float a = pb * g[t];
                    if (isfinite(a)) dv[t] += a;
                    float b = gs * qr[t] * c->sm_scale;
                    if (isfinite(b)) dk[t] += b;
                }
            }
        }
    free(invN); free(accdO); free(active);
}

/* The reference notebook's top-k-only "stable" operator
 * (AdaSplashNotebook.ipynb file lines 303-375, stable_entmax_threshold, and
 * 376-450, stable_splash_kernel), from each row's top-k lists as
 * asa_oracle_tau_mask produces them (with ref_tile_load = 0: the notebook
 * kernel reads K rows directly): α clamped to [1.01, 3]; τ by five
 * bisection steps from [(α-1)s_min - 1, (α-1)s_max + 1] with the |f| < 1e-4
 * exit and the τ clamp; p_j = u_j^{1/(α-1)} for u_j > EPS, normalised by
 * max(Σp, EPS), a non-finite weight -> 1/k; O = Σ_j p_j V[key_j] in j order
 * (one FMA per step), non-finite -> 0.  tau_coef receives the weight of the
 * upper start (or of the upper τ clamp) in the final τ. */
void asa_oracle_stable_forward(const asa_oracle_cfg* c, const float* V, const float* topv,
                               const int32_t* topi, float* O, float* tau_out, float* weights,
                               float* tau_coef) {
    const int k = c->k_keep, d = c->d;
    const float alpha = fmaxf(1.01f, fminf(c->alpha, 3.0f));
    const float am1 = alpha - 1.0f;
    const float inv = 1.0f / am1;
    #pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)c->BH * c->NQ; ++r) {
        const float* s = topv + (size_t)r * k;
        const float s_max = s[0], s_min = s[k - 1];
        float lo = fmaf(am1, s_min, -1.0f), hi = fmaf(am1, s_max, 1.0f);
        float clo = 0.0f, chi = 1.0f;
        float tau = 0.5f * (lo + hi), ct = 0.5f;
        for (int it = 0; it < ASA_MAX_HALLEY; ++it) {
            float f = -1.0f;
            for (int j = 0; j < k; ++j) {
                const float u = fmaf(am1, s[j], -tau);
                if (u <= 0.0f) break;
                float up = powf(fmaxf(u, ASA_EPS), inv);
                if (isnan(up) || isinf(up)) up = 0.0f;
                f += up;
            }
            if (fabsf(f) < 1e-4f) break;
            if (f > 0.0f) { lo = tau; clo = ct; } else { hi = tau; chi = ct; }
            tau = 0.5f * (lo + hi);
            ct = 0.5f * (clo + chi);
            const float tmin = fmaf(s_min, am1, -10.0f), tmax = fmaf(s_max, am1, 10.0f);
            if (tau < tmin) { tau = tmin; ct = 0.0f; }
            if (tau > tmax) { tau = tmax; ct = 1.0f; }
        }
        float p[ASA_KMAX], norm = 0.0f;
        for (int j = 0; j < k; ++j) {
            const float u = fmaf(am1, s[j], -tau);
            float pj = (u > ASA_EPS) ? powf(u, inv) : 0.0f;
            if (isnan(pj) || isinf(pj)) pj = 0.0f;
            p[j] = pj;
            norm += pj;
        }
        norm = fmaxf(norm, ASA_EPS);
        for (int j = 0; j < k; ++j) {
            p[j] /= norm;
            if (isnan(p[j]) || isinf(p[j])) p[j] = 1.0f / k;
            weights[(size_t)r * k + j] = p[j];
        }
        tau_out[r] = tau;
        tau_coef[r] = ct;
        const size_t bh = (size_t)r / c->NQ;
        for (int t = 0; t < d; ++t) {
            float acc = 0.0f;
            for (int j = 0; j < k; ++j) {
                const int key = topi[(size_t)r * k + j];
                if (key >= 0) acc = fmaf(p[j], V[(bh * c->NK + key) * d + t], acc);
            }
            O[(size_t)r * d + t] = (isnan(acc) || isinf(acc)) ? 0.0f : acc;
        }
    }
}
