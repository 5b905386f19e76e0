/*
 * CPU restatement of the reference selective-scan math -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, never the product: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference legs may load it.  The product path is the
 * CUDA library under ssm_mamba_b200/ and fails loudly when that library is missing.
 *
 * It is included twice by scan_ref.c, once with REAL=double (the parity oracle) and
 * once with REAL=float (the timed CPU baseline).  Every function restates the
 * reference algorithm line by line; the citations are paths inside the reference
 * project (nmquan1503/ssm-mamba):
 *
 *   forward  : csrc/selective_scan/forward_kernel.cu:136-243
 *   backward : csrc/selective_scan/backward_kernel.cu:212-452
 *   update   : csrc/selective_update/kernel.cu:45-77
 *   gate     : modules/mamba.py:182 (out * silu(gate)), fused here when z != NULL
 *   conv1d   : modules/mamba.py:37-44, 114-139, 203-213 (the causal depthwise conv and SiLU
 *              in front of the scan)
 *
 * Layouts (all contiguous, row-major):
 *   u, delta, z, dout, out, y, du, ddelta, dz : (batch, dim, seqlen)
 *   A, dA                                     : (dim, dstate)
 *   Bm, Cm, dB, dC                            : (batch, dstate, seqlen)
 *   Dv, bias, dD, dbias                       : (dim)
 *   h_init, h_last, dh_last, dh_init          : (batch, dim, dstate)
 *   ckpt                                      : (batch, dim, nchunks, 2*dstate), pairs
 *                                               (running product of decays, state) at the
 *                                               end of every 128-token chunk, exactly the
 *                                               reference's `h` (selective_scan.cpp:271-274)
 *   length                                    : (batch) int64, or NULL for full length
 */

#define CAT2(a, b) a##b
#define CAT(a, b) CAT2(a, b)
#define FN(name) CAT(name, SUFFIX)

/* softplus with the reference's threshold of 20 (forward_kernel.cu:155-159). */
static inline REAL FN(softplus_)(REAL x) {
    return x <= (REAL)20 ? LOG1P(EXP(x)) : x;
}

static inline REAL FN(sigmoid_)(REAL x) {
    return (REAL)1 / ((REAL)1 + EXP(-x));
}

/* Clamp a length entry to [0, L].  The reference does not clamp; outside that range
 * its backward reads past the end of the row (backward_kernel.cu:242-246). */
static inline int64_t FN(clamp_len_)(const int64_t* length, int64_t b, int64_t L) {
    if (!length) return L;
    int64_t v = length[b];
    if (v < 0) v = 0;
    if (v > L) v = L;
    return v;
}

/* Position t of a batch row is an identity step (decay 1, input 0) when it lies in the
 * padding: right padding masks t >= len, left padding masks t < L - len
 * (forward_kernel.cu:196-205, backward_kernel.cu:299-326). */
static inline int FN(masked_)(int64_t t, int64_t len, int64_t L, int padding_right) {
    return padding_right ? (t >= len) : (t < L - len || t >= L);
}

/*
 * Forward.  delta_t = softplus(delta_raw_t + bias) (or delta_raw + bias when softplus
 * is 0), decay = exp(delta*A), input = delta*u*B, h_t = decay*h_{t-1} + input,
 * y_t = D*u_t + sum_n C_t,n h_t,n, out_t = y_t * silu(z_t) when z is given.
 */
int FN(oracle_scan_fwd_)(
    int64_t Bsz, int64_t Dn, int64_t L, int64_t N,
    const REAL* u, const REAL* delta, const REAL* A, const REAL* Bm, const REAL* Cm,
    const REAL* Dv, const REAL* z, const REAL* bias, const REAL* h_init,
    const int64_t* length, int padding_right, int softplus,
    REAL* out, REAL* y, REAL* ckpt, REAL* h_last)
{
    const int64_t nck = (L + 127) / 128;
    if (N < 1 || N > 256) return 2;
    #pragma omp parallel for schedule(dynamic, 4)
    for (int64_t bd = 0; bd < Bsz * Dn; bd++) {
        const int64_t b = bd / Dn, d = bd % Dn;
        const int64_t len = FN(clamp_len_)(length, b, L);
        REAL h[256], P[256];
        for (int64_t n = 0; n < N; n++) {
            h[n] = h_init ? h_init[bd * N + n] : (REAL)0;
            P[n] = (REAL)1;
        }
        const REAL Dd = Dv ? Dv[d] : (REAL)0;
        const REAL bi = bias ? bias[d] : (REAL)0;
        for (int64_t t = 0; t < L; t++) {
            const int64_t i = bd * L + t;
            const REAL x = delta[i] + bi;
            const REAL dt = softplus ? FN(softplus_)(x) : x;
            const REAL du_ = dt * u[i];
            const int m = FN(masked_)(t, len, L, padding_right);
            REAL acc = Dd * u[i];
            for (int64_t n = 0; n < N; n++) {
                REAL a = (REAL)1, bb = (REAL)0;
                if (!m) {
                    a = EXP(dt * A[d * N + n]);
                    bb = du_ * Bm[(b * N + n) * L + t];
                }
                h[n] = a * h[n] + bb;
                P[n] *= a;
                acc += Cm[(b * N + n) * L + t] * h[n];
            }
            if (y) y[i] = acc;
            out[i] = z ? acc * z[i] * FN(sigmoid_)(z[i]) : acc;
            if (ckpt && ((t % 128) == 127 || t == L - 1)) {
                REAL* c = ckpt + (bd * nck + t / 128) * 2 * N;
                for (int64_t n = 0; n < N; n++) { c[2 * n] = P[n]; c[2 * n + 1] = h[n]; }
            }
        }
        if (h_last)
            for (int64_t n = 0; n < N; n++) h_last[bd * N + n] = h[n];
    }
    return 0;
}

/*
 * Backward, restating backward_kernel.cu:212-452 including its length handling:
 *  - chunks whose first token is >= len are skipped: du = ddelta = 0 there and the
 *    state gradient restarts from dh_last (:225-239);
 *  - when L % 128 != 0 the loads are zero-filled from token len on (:242-246, :279-291);
 *    when L % 128 == 0 they are not (vector loads, common.h:288-293);
 *  - padded positions are identity steps with no C*dout injection (:299-326);
 *  - ddelta and dA only take tokens t < len (:374-380); dB/dC only get t < len (:389-400);
 *  - dh_init = decay_0 * dh_0 (:368-370).
 * The forward recompute inside a chunk starts from the forward's saved chunk state
 * (ckpt), as the reference does (:345-353).
 * With z given, dout is first multiplied by silu(z) and dz = dout*y*silu'(z); this path
 * is only used with length == NULL.
 */
int FN(oracle_scan_bwd_)(
    int64_t Bsz, int64_t Dn, int64_t L, int64_t N,
    const REAL* u, const REAL* delta, const REAL* A, const REAL* Bm, const REAL* Cm,
    const REAL* Dv, const REAL* z, const REAL* bias, const REAL* h_init,
    const int64_t* length, int padding_right, int softplus,
    const REAL* ckpt, const REAL* y, const REAL* dout, const REAL* dh_last,
    REAL* du, REAL* ddelta, REAL* dA, REAL* dB, REAL* dC,
    REAL* dD, REAL* dbias, REAL* dz, REAL* dh_init)
{
    const int64_t nck = (L + 127) / 128;
    const int divisible = (L % 128) == 0;
    if (N < 1 || N > 256) return 2;
    int nthr = 1;
#ifdef _OPENMP
    nthr = omp_get_max_threads();
#endif
    /* Per-thread accumulators keep the reductions deterministic for a fixed thread count. */
    REAL* accBC = (REAL*)calloc((size_t)nthr * 2 * Bsz * N * L, sizeof(REAL));
    REAL* accA = (REAL*)calloc((size_t)nthr * Dn * N, sizeof(REAL));
    REAL* accD = (REAL*)calloc((size_t)nthr * Dn * 2, sizeof(REAL));
    if (!accBC || !accA || !accD) { free(accBC); free(accA); free(accD); return 1; }

    #pragma omp parallel
    {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        REAL* tB = accBC + (size_t)tid * 2 * Bsz * N * L;
        REAL* tC = tB + Bsz * N * L;
        REAL* tA = accA + (size_t)tid * Dn * N;
        REAL* tD = accD + (size_t)tid * Dn * 2;
        /* scratch for one chunk, on the heap: 2 x 128 x N values per thread */
        REAL* hs = (REAL*)malloc(sizeof(REAL) * 128 * (size_t)N);
        REAL* as_ = (REAL*)malloc(sizeof(REAL) * 128 * (size_t)N);
        REAL dlt[128], dlu[128], uu[128], dd[128], xr[128];
        REAL g[256], anext[256];

        #pragma omp for schedule(dynamic, 4)
        for (int64_t bd = 0; bd < Bsz * Dn; bd++) {
            const int64_t b = bd / Dn, d = bd % Dn;
            const int64_t len = FN(clamp_len_)(length, b, L);
            const int64_t Lload = divisible ? L : len;
            const REAL Dd = Dv ? Dv[d] : (REAL)0;
            const REAL bi = bias ? bias[d] : (REAL)0;
            for (int64_t n = 0; n < N; n++) {
                g[n] = dh_last ? dh_last[bd * N + n] : (REAL)0;
                anext[n] = (REAL)1;
            }
            int wrote_dh_init = 0;
            for (int64_t c = nck - 1; c >= 0; c--) {
                const int64_t t0 = c * 128;
                const int64_t t1 = (t0 + 128 < L) ? t0 + 128 : L;
                if (t0 >= len) {
                    for (int64_t t = t0; t < t1; t++) {
                        du[bd * L + t] = 0; ddelta[bd * L + t] = 0;
                        if (dz) dz[bd * L + t] = 0;
                    }
                    for (int64_t n = 0; n < N; n++) {
                        g[n] = dh_last ? dh_last[bd * N + n] : (REAL)0;
                        anext[n] = (REAL)1;
                    }
                    continue;
                }
                /* loads and per-token prologue */
                for (int64_t t = t0; t < t1; t++) {
                    const int64_t i = bd * L + t, k = t - t0;
                    const int ld = t < Lload;
                    const REAL uv = ld ? u[i] : 0, dr = ld ? delta[i] : 0;
                    REAL dv = ld ? dout[i] : 0;
                    if (z) {
                        const REAL s = FN(sigmoid_)(z[i]);
                        const REAL sz = z[i] * s;
                        dz[i] = dv * y[i] * s * ((REAL)1 + z[i] * ((REAL)1 - s));
                        dv = dv * sz;
                    }
                    const REAL x = dr + bi;
                    xr[k] = x;
                    dlt[k] = softplus ? FN(softplus_)(x) : x;
                    dlu[k] = dlt[k] * uv;
                    uu[k] = uv;
                    dd[k] = dv;
                }
                /* forward recompute from the saved state of the previous chunk */
                for (int64_t n = 0; n < N; n++) {
                    REAL hp = (c == 0) ? (h_init ? h_init[bd * N + n] : (REAL)0)
                                       : ckpt[(bd * nck + c - 1) * 2 * N + 2 * n + 1];
                    for (int64_t t = t0; t < t1; t++) {
                        const int64_t k = t - t0;
                        const int m = FN(masked_)(t, len, L, padding_right);
                        const REAL Bv = (t < Lload) ? Bm[(b * N + n) * L + t] : 0;
                        REAL a = 1, bb = 0;
                        if (!m) { a = EXP(dlt[k] * A[d * N + n]); bb = dlu[k] * Bv; }
                        hp = a * hp + bb;
                        hs[k * N + n] = hp;
                        as_[k * N + n] = a;
                    }
                }
                /* reverse pass */
                for (int64_t t = t1 - 1; t >= t0; t--) {
                    const int64_t i = bd * L + t, k = t - t0;
                    const int m = FN(masked_)(t, len, L, padding_right);
                    const int valid = t < len;
                    REAL s1 = 0, s2 = 0;
                    for (int64_t n = 0; n < N; n++) {
                        const REAL Bv = (t < Lload) ? Bm[(b * N + n) * L + t] : 0;
                        const REAL Cv = (t < Lload) ? Cm[(b * N + n) * L + t] : 0;
                        const REAL inj = m ? 0 : dd[k] * Cv;
                        const REAL G = inj + anext[n] * g[n];
                        g[n] = G;
                        anext[n] = as_[k * N + n];
                        const REAL h = hs[k * N + n];
                        const REAL q = h - dlu[k] * Bv;
                        s1 += G * Bv;
                        if (valid) {
                            s2 += G * A[d * N + n] * q;
                            tA[d * N + n] += G * dlt[k] * q;
                            tB[(b * N + n) * L + t] += G * dlu[k];
                            tC[(b * N + n) * L + t] += dd[k] * h;
                        }
                    }
                    du[i] = Dd * dd[k] + dlt[k] * s1;
                    REAL ddl = valid ? uu[k] * s1 + s2 : 0;
                    if (softplus && xr[k] <= (REAL)20) ddl *= FN(sigmoid_)(xr[k]);
                    ddelta[i] = ddl;
                    tD[2 * d] += dd[k] * uu[k];
                    tD[2 * d + 1] += ddl;
                }
                if (c == 0 && dh_init) {
                    for (int64_t n = 0; n < N; n++) dh_init[bd * N + n] = anext[n] * g[n];
                    wrote_dh_init = 1;
                }
            }
            /* len == 0: every chunk was skipped; the reference leaves dh_init unwritten,
             * here it is the gradient that passes through the all-identity row. */
            if (dh_init && !wrote_dh_init)
                for (int64_t n = 0; n < N; n++)
                    dh_init[bd * N + n] = dh_last ? dh_last[bd * N + n] : (REAL)0;
        }
        free(hs);
        free(as_);
    }
    /* deterministic reductions in thread order */
    memset(dA, 0, sizeof(REAL) * Dn * N);
    memset(dB, 0, sizeof(REAL) * Bsz * N * L);
    memset(dC, 0, sizeof(REAL) * Bsz * N * L);
    if (dD) memset(dD, 0, sizeof(REAL) * Dn);
    if (dbias) memset(dbias, 0, sizeof(REAL) * Dn);
    for (int th = 0; th < nthr; th++) {
        const REAL* tB = accBC + (size_t)th * 2 * Bsz * N * L;
        const REAL* tC = tB + Bsz * N * L;
        for (int64_t j = 0; j < Bsz * N * L; j++) { dB[j] += tB[j]; dC[j] += tC[j]; }
        for (int64_t j = 0; j < Dn * N; j++) dA[j] += accA[(size_t)th * Dn * N + j];
        for (int64_t j = 0; j < Dn; j++) {
            if (dD) dD[j] += accD[(size_t)th * Dn * 2 + 2 * j];
            if (dbias) dbias[j] += accD[(size_t)th * Dn * 2 + 2 * j + 1];
        }
    }
    free(accBC); free(accA); free(accD);
    return 0;
}

/*
 * One decode step, restating selective_update/kernel.cu:45-77:
 * h' = exp(delta*A)*h + delta*u*B, out = sum_n C*h' + D*u, with the optional gate and
 * the optional softplus of the new selective_state_update surface.  h_out may alias h_in.
 */
int FN(oracle_state_update_)(
    int64_t Bsz, int64_t Dn, int64_t N,
    const REAL* u, const REAL* delta, const REAL* A, const REAL* Bm, const REAL* Cm,
    const REAL* Dv, const REAL* z, const REAL* bias, int softplus,
    const REAL* h_in, REAL* h_out, REAL* out)
{
    #pragma omp parallel for schedule(static)
    for (int64_t bd = 0; bd < Bsz * Dn; bd++) {
        const int64_t b = bd / Dn, d = bd % Dn;
        const REAL x = delta[bd] + (bias ? bias[d] : (REAL)0);
        const REAL dt = softplus ? FN(softplus_)(x) : x;
        REAL acc = (Dv ? Dv[d] : (REAL)0) * u[bd];
        for (int64_t n = 0; n < N; n++) {
            const REAL hn = EXP(dt * A[d * N + n]) * h_in[bd * N + n] + dt * u[bd] * Bm[b * N + n];
            h_out[bd * N + n] = hn;
            acc += Cm[b * N + n] * hn;
        }
        out[bd] = z ? acc * z[bd] * FN(sigmoid_)(z[bd]) : acc;
    }
    return 0;
}

/*
 * Causal depthwise conv1d + optional SiLU, restating the reference's Mamba module:
 *   prefill  silu(nn.Conv1d(dim, dim, width, groups=dim, padding=width-1)(x)[..., :L])
 *            (modules/mamba.py:37-44, 137-139): out[t] = bias + sum_k w[k] x[t-(width-1)+k]
 *   context  the last width-1 inputs before length[b], zero before the row start
 *            (modules/mamba.py:114-133)
 *   decode   window = cat(context, x); out = silu(sum_k window[k] w[k] + bias); the context
 *            shifts by one (modules/mamba.py:203-213)
 * Layouts: x, out, dout, dx (batch, dim, L); w, dw (dim, width); bias, dbias (dim);
 * state (batch, dim, width-1).  The backward is the exact gradient of the prefill.
 */
int FN(oracle_conv1d_fwd_)(int64_t Bsz, int64_t Dn, int64_t L, int64_t K, const REAL* x, const REAL* w,
                           const REAL* bias, int silu, REAL* out)
{
    #pragma omp parallel for schedule(static)
    for (int64_t bd = 0; bd < Bsz * Dn; bd++) {
        const int64_t d = bd % Dn;
        for (int64_t t = 0; t < L; t++) {
            REAL acc = bias ? bias[d] : (REAL)0;
            for (int64_t k = 0; k < K; k++) {
                const int64_t s = t - (K - 1) + k;
                if (s >= 0) acc += w[d * K + k] * x[bd * L + s];
            }
            out[bd * L + t] = silu ? acc * FN(sigmoid_)(acc) : acc;
        }
    }
    return 0;
}

int FN(oracle_conv1d_bwd_)(int64_t Bsz, int64_t Dn, int64_t L, int64_t K, const REAL* x, const REAL* w,
                           const REAL* bias, int silu, const REAL* dout, REAL* dx, REAL* dw, REAL* dbias)
{
    REAL* g = (REAL*)malloc(sizeof(REAL) * Bsz * Dn * L);
    if (!g) return 3;
    #pragma omp parallel for schedule(static)
    for (int64_t bd = 0; bd < Bsz * Dn; bd++) {
        const int64_t d = bd % Dn;
        for (int64_t t = 0; t < L; t++) {
            REAL pre = bias ? bias[d] : (REAL)0;
            for (int64_t k = 0; k < K; k++) {
                const int64_t s = t - (K - 1) + k;
                if (s >= 0) pre += w[d * K + k] * x[bd * L + s];
            }
            REAL gi = dout[bd * L + t];
            if (silu) {
                const REAL sg = FN(sigmoid_)(pre);
                gi *= sg * ((REAL)1 + pre * ((REAL)1 - sg));
            }
            g[bd * L + t] = gi;
        }
        for (int64_t t = 0; t < L; t++) {
            REAL acc = 0;
            for (int64_t k = 0; k < K; k++) {
                const int64_t s = t + (K - 1) - k;
                if (s < L) acc += w[d * K + k] * g[bd * L + s];
            }
            dx[bd * L + t] = acc;
        }
    }
    #pragma omp parallel for schedule(static)
    for (int64_t d = 0; d < Dn; d++) {
        REAL db = 0;
        for (int64_t k = 0; k < K; k++) {
            REAL acc = 0;
            for (int64_t b = 0; b < Bsz; b++)
                for (int64_t t = 0; t < L; t++) {
                    const int64_t s = t - (K - 1) + k;
                    if (s >= 0) acc += g[(b * Dn + d) * L + t] * x[(b * Dn + d) * L + s];
                }
            dw[d * K + k] = acc;
        }
        for (int64_t b = 0; b < Bsz; b++)
            for (int64_t t = 0; t < L; t++) db += g[(b * Dn + d) * L + t];
        if (dbias) dbias[d] = db;
    }
    free(g);
    return 0;
}

int FN(oracle_conv1d_state_)(int64_t Bsz, int64_t Dn, int64_t L, int64_t K, const REAL* x,
                             const int64_t* length, REAL* state)
{
    for (int64_t bd = 0; bd < Bsz * Dn; bd++) {
        const int64_t len = FN(clamp_len_)(length, bd / Dn, L);
        for (int64_t j = 0; j < K - 1; j++) {
            const int64_t t = len - (K - 1) + j;
            state[bd * (K - 1) + j] = t >= 0 ? x[bd * L + t] : (REAL)0;
        }
    }
    return 0;
}

int FN(oracle_conv1d_update_)(int64_t Bsz, int64_t Dn, int64_t K, const REAL* x, REAL* state, const REAL* w,
                              const REAL* bias, int silu, REAL* out)
{
    for (int64_t bd = 0; bd < Bsz * Dn; bd++) {
        const int64_t d = bd % Dn;
        REAL acc = bias ? bias[d] : (REAL)0;
        for (int64_t k = 0; k < K - 1; k++) acc += w[d * K + k] * state[bd * (K - 1) + k];
        acc += w[d * K + K - 1] * x[bd];
        for (int64_t k = 0; k + 1 < K - 1; k++) state[bd * (K - 1) + k] = state[bd * (K - 1) + k + 1];
        state[bd * (K - 1) + K - 2] = x[bd];
        out[bd] = silu ? acc * FN(sigmoid_)(acc) : acc;
    }
    return 0;
}

#undef FN
