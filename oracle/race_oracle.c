/*
 * race_oracle.c -- CPU oracle for the causal RACE attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
 * legs may load it.  The CUDA library (race_attention_b200/csrc) never calls it
 * and the Python operator surface fails loudly instead of falling back to it.
 *
 * It restates, in plain C with double-precision accumulation, the reference's
 * own algorithm (paths relative to the reference project root):
 *
 *   oracle_soft_hash      scaling/race_common.py:36-73   (soft_hash_probs)
 *   oracle_soft_hash_bwd  autograd of scaling/race_common.py:56-72
 *   oracle_race_fwd       scaling/race_common.py:76-90   (race_prefix_ref),
 *                         extended with an optional carried-in state (A0,B0)
 *                         so the same routine is the decode-step and the
 *                         sequence-shard oracle
 *   oracle_race_bwd       scaling/race_causal_cpu.py:52-72 composed with
 *                         kernels/cpu/race_pref.cpp:104-220
 *                         (race_prefix_mean_flat_bw), restated per (n,s)
 *                         stream without materialising V expanded x S, and
 *                         extended with an incoming suffix gradient (gA, gB)
 *                         for the final state, which is what a later sequence
 *                         shard sends back to an earlier one
 *
 * Layouts are the reference's: Q/K/V/out [N,T,D]; probs [N,T,S] with
 * S = L*R, R = 2^P, bucket index s = l*R + r (table-outer, corner-inner);
 * planes_T [D, L*P] with column j = l*P + p; corner r has hyperplane sign
 * +1 for bit p iff bit (P-1-p) of r is set (itertools.product order,
 * scaling/race_common.py:30-32).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

int oracle_abi_version(void) { return 1; }

static inline double corner_sign(long r, long p, long P)
{
    return ((r >> (P - 1 - p)) & 1) ? 1.0 : -1.0;
}

/* probs[n,t,l*R+r] = softmax_r( sum_p tanh(x.planes_T[:,l*P+p]) * scale * sign(p,r) ) */
void oracle_soft_hash(const double *X, long N, long T, long D,
                      const double *planes_T, long L, long P, double logit_scale,
                      double *probs)
{
    const long LP = L * P, R = 1L << P, S = L * R;
    double *a = (double *)malloc(sizeof(double) * LP);
    double *lg = (double *)malloc(sizeof(double) * R);
    for (long n = 0; n < N; ++n)
        for (long t = 0; t < T; ++t) {
            const double *x = X + (n * T + t) * D;
            double *pr = probs + (n * T + t) * S;
            for (long j = 0; j < LP; ++j) {
                double acc = 0.0;
                for (long d = 0; d < D; ++d) acc += x[d] * planes_T[d * LP + j];
                a[j] = tanh(acc) * logit_scale;
            }
            for (long l = 0; l < L; ++l) {
                double mx = -INFINITY;
                for (long r = 0; r < R; ++r) {
                    double v = 0.0;
                    for (long p = 0; p < P; ++p) v += a[l * P + p] * corner_sign(r, p, P);
                    lg[r] = v;
                    if (v > mx) mx = v;
                }
                double z = 0.0;
                for (long r = 0; r < R; ++r) { lg[r] = exp(lg[r] - mx); z += lg[r]; }
                for (long r = 0; r < R; ++r) pr[l * R + r] = lg[r] / z;
            }
        }
    free(a);
    free(lg);
}

/* dX = d/dX < dprobs, soft_hash(X) >  (planes are buffers: no gradient for them). */
void oracle_soft_hash_bwd(const double *X, long N, long T, long D,
                          const double *planes_T, long L, long P, double logit_scale,
                          const double *dprobs, double *dX)
{
    const long LP = L * P, R = 1L << P, S = L * R;
    double *th = (double *)malloc(sizeof(double) * LP);
    double *da = (double *)malloc(sizeof(double) * LP);
    double *pr = (double *)malloc(sizeof(double) * R);
    for (long n = 0; n < N; ++n)
        for (long t = 0; t < T; ++t) {
            const double *x = X + (n * T + t) * D;
            const double *g = dprobs + (n * T + t) * S;
            double *dx = dX + (n * T + t) * D;
            for (long j = 0; j < LP; ++j) {
                double acc = 0.0;
                for (long d = 0; d < D; ++d) acc += x[d] * planes_T[d * LP + j];
                th[j] = tanh(acc);
            }
            for (long l = 0; l < L; ++l) {
                double mx = -INFINITY;
                for (long r = 0; r < R; ++r) {
                    double v = 0.0;
                    for (long p = 0; p < P; ++p) v += th[l * P + p] * logit_scale * corner_sign(r, p, P);
                    pr[r] = v;
                    if (v > mx) mx = v;
                }
                double z = 0.0;
                for (long r = 0; r < R; ++r) { pr[r] = exp(pr[r] - mx); z += pr[r]; }
                double c = 0.0;
                for (long r = 0; r < R; ++r) { pr[r] /= z; c += pr[r] * g[l * R + r]; }
                for (long p = 0; p < P; ++p) {
                    double acc = 0.0;
                    for (long r = 0; r < R; ++r)
                        acc += pr[r] * (g[l * R + r] - c) * corner_sign(r, p, P);
                    da[l * P + p] = acc;
                }
            }
            for (long d = 0; d < D; ++d) {
                double acc = 0.0;
                for (long j = 0; j < LP; ++j)
                    acc += da[j] * logit_scale * (1.0 - th[j] * th[j]) * planes_T[d * LP + j];
                dx[d] = acc;
            }
        }
    free(th);
    free(da);
    free(pr);
}

/*
 * out[n,t,:] = sum_s pq[n,t,s] * B_t[n,s,:] / (A_t[n,s] + eps)
 * A_t = A0 + sum_{tau<=t} pk[tau],  B_t = B0 + sum_{tau<=t} pk[tau] * V[tau]
 * A0/B0 may be NULL (zero state).  A_fin/B_fin may be NULL.
 */
void oracle_race_fwd(const double *pk, const double *pq, const double *V,
                     long N, long T, long S, long D, double eps,
                     const double *A0, const double *B0,
                     double *out, double *A_fin, double *B_fin)
{
    double *A = (double *)malloc(sizeof(double) * S);
    double *B = (double *)malloc(sizeof(double) * S * D);
    for (long n = 0; n < N; ++n) {
        for (long s = 0; s < S; ++s) A[s] = A0 ? A0[n * S + s] : 0.0;
        for (long i = 0; i < S * D; ++i) B[i] = B0 ? B0[n * S * D + i] : 0.0;
        for (long t = 0; t < T; ++t) {
            const double *k = pk + (n * T + t) * S;
            const double *q = pq + (n * T + t) * S;
            const double *v = V + (n * T + t) * D;
            double *o = out + (n * T + t) * D;
            for (long d = 0; d < D; ++d) o[d] = 0.0;
            for (long s = 0; s < S; ++s) {
                A[s] += k[s];
                double *b = B + s * D;
                for (long d = 0; d < D; ++d) b[d] += k[s] * v[d];
                const double w = q[s] / (A[s] + eps);
                for (long d = 0; d < D; ++d) o[d] += w * b[d];
            }
        }
        if (A_fin) memcpy(A_fin + n * S, A, sizeof(double) * S);
        if (B_fin) memcpy(B_fin + n * S * D, B, sizeof(double) * S * D);
    }
    free(A);
    free(B);
}

/*
 * Exact gradients of oracle_race_fwd for the loss
 *     sum_t dO_t . out_t  +  <gA_in, A_final> + <gB_in, B_final>
 * (gA_in [N,S] / gB_in [N,S,D] may be NULL = 0).  Outputs dpk, dpq [N,T,S],
 * dV [N,T,D] and, when non-NULL, dA0 [N,S], dB0 [N,S,D] (gradient of the
 * carried-in state).  Per (n,s) stream this is race_prefix_mean_flat_bw:
 * pass 1 runs forward over t keeping 1/(A+eps) and
 * alpha_t = -(1/(A+eps))^2 * (pq_t dO_t . B_t); pass 2 runs backward
 * accumulating beta = sum_{t'>=t} pq dO /(A+eps) and alpha_suf, giving
 * dpk = alpha_suf + beta . v_t and the V contribution pk_t * beta.
 */
void oracle_race_bwd(const double *pk, const double *pq, const double *V, const double *dO,
                     long N, long T, long S, long D, double eps,
                     const double *A0, const double *B0,
                     const double *gA_in, const double *gB_in,
                     double *dpk, double *dpq, double *dV,
                     double *dA0, double *dB0)
{
    double *invA = (double *)malloc(sizeof(double) * (T > 0 ? T : 1));
    double *alpha = (double *)malloc(sizeof(double) * (T > 0 ? T : 1));
    double *B = (double *)malloc(sizeof(double) * D);
    double *beta = (double *)malloc(sizeof(double) * D);
    for (long i = 0; i < N * T * D; ++i) dV[i] = 0.0;
    for (long n = 0; n < N; ++n) {
        for (long s = 0; s < S; ++s) {
            double A = A0 ? A0[n * S + s] : 0.0;
            for (long d = 0; d < D; ++d) B[d] = B0 ? B0[(n * S + s) * D + d] : 0.0;
            for (long t = 0; t < T; ++t) {
                const double w = pk[(n * T + t) * S + s];
                const double q = pq[(n * T + t) * S + s];
                const double *v = V + (n * T + t) * D;
                const double *g = dO + (n * T + t) * D;
                A += w;
                double G = 0.0;
                for (long d = 0; d < D; ++d) { B[d] += w * v[d]; G += g[d] * B[d]; }
                const double iA = 1.0 / (A + eps);
                invA[t] = iA;
                alpha[t] = -(iA * iA) * q * G;
                dpq[(n * T + t) * S + s] = G * iA;
            }
            double alpha_suf = gA_in ? gA_in[n * S + s] : 0.0;
            for (long d = 0; d < D; ++d) beta[d] = gB_in ? gB_in[(n * S + s) * D + d] : 0.0;
            for (long t = T - 1; t >= 0; --t) {
                const double w = pk[(n * T + t) * S + s];
                const double q = pq[(n * T + t) * S + s];
                const double *v = V + (n * T + t) * D;
                const double *g = dO + (n * T + t) * D;
                double *gv = dV + (n * T + t) * D;
                alpha_suf += alpha[t];
                double bv = 0.0;
                for (long d = 0; d < D; ++d) {
                    beta[d] += q * g[d] * invA[t];
                    bv += beta[d] * v[d];
                    gv[d] += w * beta[d];
                }
                dpk[(n * T + t) * S + s] = alpha_suf + bv;
            }
            if (dA0) dA0[n * S + s] = alpha_suf;
            if (dB0) for (long d = 0; d < D; ++d) dB0[(n * S + s) * D + d] = beta[d];
        }
    }
    free(invA);
    free(alpha);
    free(B);
    free(beta);
}

/*
 * ---------------------------------------------------------------------------
 * Whole-layer oracle for long sequences, one stream at a time, multithreaded
 * (OpenMP).  Same algorithm and fp64 accumulation as oracle_soft_hash +
 * oracle_race_fwd / oracle_race_bwd + oracle_soft_hash_bwd above
 * (scaling/race_common.py:36-90, scaling/race_causal_cpu.py:52-72 over
 * kernels/cpu/race_pref.cpp:104-220); only the work is split so that T in the
 * millions finishes in seconds:
 *   - soft hash and its backward: parallel over tokens;
 *   - per-bucket scans (A_t, 1/(A_t+eps), dpq, dpk): parallel over buckets s;
 *   - the D-wide sums (out, dV): parallel over d, each thread carrying the
 *     bucket states of its own d columns.
 * The [T,S] intermediates (pk, W = pq/(A+eps), 1/(A+eps), dpk, dpq) are
 * stored as float (a rounding of 6e-8 relative, far below every tolerance
 * they are used at) so that T = 4M, S = 128 needs about 10 GB of host memory;
 * every sum is accumulated in double.  Inputs are float (bf16 inputs convert
 * exactly).
 */
#include <omp.h>

static void hash_rows_f(const float *X, long T, long D, const double *planes_T, long L, long P,
                        double scale, float *probs, double *th_out /* [T,LP] or NULL */)
{
    const long LP = L * P, R = 1L << P, S = L * R;
#pragma omp parallel
    {
        double *a = (double *)malloc(sizeof(double) * LP);
        double *lg = (double *)malloc(sizeof(double) * R);
#pragma omp for schedule(static)
        for (long t = 0; t < T; ++t) {
            const float *x = X + t * D;
            for (long j = 0; j < LP; ++j) {
                double acc = 0.0;
                for (long d = 0; d < D; ++d) acc += (double)x[d] * planes_T[d * LP + j];
                const double th = tanh(acc);
                if (th_out) th_out[t * LP + j] = th;
                a[j] = th * scale;
            }
            for (long l = 0; l < L; ++l) {
                double mx = -INFINITY;
                for (long r = 0; r < R; ++r) {
                    double v = 0.0;
                    for (long p = 0; p < P; ++p) v += a[l * P + p] * corner_sign(r, p, P);
                    lg[r] = v;
                    if (v > mx) mx = v;
                }
                double z = 0.0;
                for (long r = 0; r < R; ++r) { lg[r] = exp(lg[r] - mx); z += lg[r]; }
                for (long r = 0; r < R; ++r) probs[t * S + l * R + r] = (float)(lg[r] / z);
            }
        }
        free(a);
        free(lg);
    }
}

/* dX[t] = gradient of <dprobs[t], soft_hash(X[t])>, from the token's tanh values. */
static void hash_rows_bwd_f(long T, long D, const double *planes_T, long L, long P, double scale,
                            const float *probs, const double *th, const float *dprobs, double *dX)
{
    const long LP = L * P, R = 1L << P, S = L * R;
#pragma omp parallel
    {
        double *da = (double *)malloc(sizeof(double) * LP);
#pragma omp for schedule(static)
        for (long t = 0; t < T; ++t) {
            const float *pr = probs + t * S;
            const float *g = dprobs + t * S;
            for (long l = 0; l < L; ++l) {
                double c = 0.0;
                for (long r = 0; r < R; ++r) c += (double)pr[l * R + r] * g[l * R + r];
                for (long p = 0; p < P; ++p) {
                    double acc = 0.0;
                    for (long r = 0; r < R; ++r)
                        acc += (double)pr[l * R + r] * ((double)g[l * R + r] - c) * corner_sign(r, p, P);
                    const double tj = th[t * LP + l * P + p];
                    da[l * P + p] = acc * scale * (1.0 - tj * tj);
                }
            }
            for (long d = 0; d < D; ++d) {
                double acc = 0.0;
                for (long j = 0; j < LP; ++j) acc += da[j] * planes_T[d * LP + j];
                dX[t * D + d] = acc;
            }
        }
        free(da);
    }
}

/*
 * One stream of the full layer: Q, K, V, dO [T,D] float; planes_T [D, L*P].
 * Forward: out [T,D], A_fin [S], B_fin [S,D] (any may be NULL except out).
 * Backward (when dO != NULL): dQ, dK, dV [T,D] (double).
 */
int oracle_layer_stream(const float *Q, const float *K, const float *V, const float *dO,
                        long T, long D, const double *planes_T, long L, long P,
                        double logit_scale, double eps,
                        double *out, double *A_fin, double *B_fin,
                        double *dQ, double *dK, double *dV)
{
    const long LP = L * P, S = L << P;
    float *pk = (float *)malloc(sizeof(float) * T * S);
    float *pq = (float *)malloc(sizeof(float) * T * S);   /* becomes W = pq / (A + eps) */
    float *inv = (float *)malloc(sizeof(float) * T * S);  /* 1 / (A + eps) */
    double *thK = dO ? (double *)malloc(sizeof(double) * T * LP) : NULL;
    double *thQ = dO ? (double *)malloc(sizeof(double) * T * LP) : NULL;
    if (!pk || !pq || !inv || (dO && (!thK || !thQ))) {
        free(pk); free(pq); free(inv); free(thK); free(thQ);
        return 1;
    }
    hash_rows_f(K, T, D, planes_T, L, P, logit_scale, pk, thK);
    hash_rows_f(Q, T, D, planes_T, L, P, logit_scale, pq, thQ);

    /* per bucket: A_t, 1/(A_t+eps), W */
#pragma omp parallel for schedule(static)
    for (long s = 0; s < S; ++s) {
        double A = 0.0;
        for (long t = 0; t < T; ++t) {
            A += pk[t * S + s];
            const double iv = 1.0 / (A + eps);
            inv[t * S + s] = (float)iv;
            pq[t * S + s] = (float)(pq[t * S + s] * iv);
        }
        if (A_fin) A_fin[s] = A;
    }
    /* out[t,d] = sum_s W[t,s] B_t[s,d], per column d */
#pragma omp parallel
    {
        double *B = (double *)malloc(sizeof(double) * S);
#pragma omp for schedule(dynamic, 1)
        for (long d = 0; d < D; ++d) {
            for (long s = 0; s < S; ++s) B[s] = 0.0;
            for (long t = 0; t < T; ++t) {
                const double v = V[t * D + d];
                const float *k = pk + t * S, *w = pq + t * S;
                double o = 0.0;
                for (long s = 0; s < S; ++s) {
                    B[s] += (double)k[s] * v;
                    o += (double)w[s] * B[s];
                }
                out[t * D + d] = o;
            }
            if (B_fin) for (long s = 0; s < S; ++s) B_fin[s * D + d] = B[s];
        }
        free(B);
    }
    if (!dO) {
        free(pk); free(pq); free(inv);
        return 0;
    }
    float *dpk = (float *)malloc(sizeof(float) * T * S);
    float *dpq = (float *)malloc(sizeof(float) * T * S);
    if (!dpk || !dpq) {
        free(pk); free(pq); free(inv); free(thK); free(thQ); free(dpk); free(dpq);
        return 1;
    }
    /* per bucket s: G_t = dO_t . B_t[s], dpq = G/(A+eps), alpha_t = -W G/(A+eps);
     * then backwards: gA = sum_{t'>=t} alpha, gB = sum_{t'>=t} W dO, dpk = gA + V.gB */
    int fail = 0;
#pragma omp parallel
    {
        double *B = (double *)malloc(sizeof(double) * D);
        double *beta = (double *)malloc(sizeof(double) * D);
        double *alpha = (double *)malloc(sizeof(double) * T);
        if (!B || !beta || !alpha) {
#pragma omp atomic write
            fail = 1;
        }
#pragma omp for schedule(dynamic, 1)
        for (long s = 0; s < S; ++s) {
            if (fail) continue;
            for (long d = 0; d < D; ++d) B[d] = 0.0;
            for (long t = 0; t < T; ++t) {
                const double w = pk[t * S + s];
                double G = 0.0;
                for (long d = 0; d < D; ++d) {
                    B[d] += w * V[t * D + d];
                    G += (double)dO[t * D + d] * B[d];
                }
                const double iv = inv[t * S + s];
                dpq[t * S + s] = (float)(G * iv);
                alpha[t] = -(double)pq[t * S + s] * G * iv;
            }
            double gA = 0.0;
            for (long d = 0; d < D; ++d) beta[d] = 0.0;
            for (long t = T - 1; t >= 0; --t) {
                const double w = pq[t * S + s];
                gA += alpha[t];
                double bv = 0.0;
                for (long d = 0; d < D; ++d) {
                    beta[d] += w * dO[t * D + d];
                    bv += beta[d] * V[t * D + d];
                }
                dpk[t * S + s] = (float)(gA + bv);
            }
        }
        free(B); free(beta); free(alpha);
    }
    if (!fail) {
        /* dV[t,d] = sum_s pk[t,s] gB_t[s,d], per column d */
#pragma omp parallel
        {
            double *beta = (double *)malloc(sizeof(double) * S);
#pragma omp for schedule(dynamic, 1)
            for (long d = 0; d < D; ++d) {
                for (long s = 0; s < S; ++s) beta[s] = 0.0;
                for (long t = T - 1; t >= 0; --t) {
                    const double g = dO[t * D + d];
                    const float *k = pk + t * S, *w = pq + t * S;
                    double acc = 0.0;
                    for (long s = 0; s < S; ++s) {
                        beta[s] += (double)w[s] * g;
                        acc += (double)k[s] * beta[s];
                    }
                    dV[t * D + d] = acc;
                }
            }
            free(beta);
        }
        /* back to the probabilities of the soft hash: pq = W (A + eps) */
#pragma omp parallel for schedule(static)
        for (long i = 0; i < T * S; ++i) pq[i] = (float)((double)pq[i] / (double)inv[i]);
        hash_rows_bwd_f(T, D, planes_T, L, P, logit_scale, pq, thQ, dpq, dQ);
        hash_rows_bwd_f(T, D, planes_T, L, P, logit_scale, pk, thK, dpk, dK);
    }
    free(pk); free(pq); free(inv); free(thK); free(thQ); free(dpk); free(dpq);
    return fail;
}
