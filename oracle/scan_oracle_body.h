/*
 * CPU restatement of the reference's scalar selective-scan recurrences.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is compiled into liboracle.so, which
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load as the
 * checker.  Nothing in the armhackathon_b200 package links or calls it.
 *
 * Included twice by scan_oracle.c, once with T=float (suffix _f32, the
 * reference's production element type and the CPU baseline) and once with
 * T=double (suffix _f64, the parity oracle).  Every function follows one
 * reference function line by line; the citation is in its comment.  Threading
 * mirrors kernel/arm-scan-core/src/parallel.rs: rows are independent, a row is
 * processed by exactly one thread (ROWS_BEGIN/ROWS_END in scan_oracle.cc),
 * so results are identical for any thread count.
 */

/* ---- numerics contract: kernel/arm-scan-core/src/float.rs:24-77 ---------- */
static inline T FN(softplus)(T x) {           /* float.rs:30-37, threshold 20 */
    return x > (T)20 ? x : LOG1P(EXP(x));
}
static inline T FN(silu)(T x) {               /* float.rs:41-43 */
    return x / ((T)1 + EXP(-x));
}
static inline T FN(sigmoid)(T x) {            /* float.rs:52-59, branch-stable */
    if (x >= (T)0) return (T)1 / ((T)1 + EXP(-x));
    T e = EXP(x);
    return e / ((T)1 + e);
}

/*
 * Mamba-1 selective scan, one (batch, channel) row.
 * Follows kernel/arm-scan-core/src/scalar.rs:11-89 (scan) and the layout
 * contract of kernel/arm-scan-core/src/lib.rs:9-16:
 *   u, delta, z, out : (batch, dim, len);  a : (dim, state)
 *   b, c : (batch, groups, state, len);    d_skip, delta_bias : (dim,)
 *   h0, last_state : (batch, dim, state)
 */
static void FN(m1_row)(const oracle_m1_dims* dm, size_t ch,
                       const T* u, const T* delta, const T* a, const T* b,
                       const T* c, const T* d_skip, const T* z,
                       const T* delta_bias, int delta_softplus, int reverse,
                       T* out, T* last_state, const T* h0, T* h) {
    const size_t dim = dm->dim, len = dm->len, state = dm->state;
    const size_t group_size = dim / dm->groups;
    const size_t bi = ch / dim, d = ch % dim;
    const T* a_row = a + d * state;
    const T bias = delta_bias ? delta_bias[d] : (T)0;
    const size_t bc_base = (bi * dm->groups + d / group_size) * state * len;
    const size_t row = ch * len;
    for (size_t n = 0; n < state; ++n) h[n] = h0 ? h0[ch * state + n] : (T)0;
    for (size_t i = 0; i < len; ++i) {
        const size_t t = reverse ? len - 1 - i : i;           /* scalar.rs:59 */
        T dt = delta[row + t] + bias;
        if (delta_softplus) dt = FN(softplus)(dt);
        const T dt_u = dt * u[row + t];
        T y = 0;
        for (size_t n = 0; n < state; ++n) {                  /* scalar.rs:68-73 */
            const size_t bc = bc_base + n * len + t;
            const T nw = EXP(dt * a_row[n]) * h[n] + dt_u * b[bc];
            h[n] = nw;
            y = y + c[bc] * nw;
        }
        if (d_skip) y = y + d_skip[d] * u[row + t];
        if (z) y = y * FN(silu)(z[row + t]);
        out[row + t] = y;
    }
    if (last_state)
        for (size_t n = 0; n < state; ++n) last_state[ch * state + n] = h[n];
}

extern "C" int FN(oracle_m1_scan)(const oracle_m1_dims* dm, const T* u, const T* delta,
                       const T* a, const T* b, const T* c, const T* d_skip,
                       const T* z, const T* delta_bias, int delta_softplus,
                       int reverse, T* out, T* last_state, const T* h0,
                       int nthreads) {
    if (!dm || !dm->batch || !dm->dim || !dm->len || !dm->state || !dm->groups ||
        dm->dim % dm->groups)
        return 2;
    const size_t state = dm->state;
    ROWS_BEGIN(dm->batch * dm->dim)
        T* h = (T*)malloc(state * sizeof(T));
        for (size_t ch = r0; ch < r1; ++ch)
            FN(m1_row)(dm, ch, u, delta, a, b, c, d_skip, z, delta_bias,
                       delta_softplus, reverse, out, last_state, h0, h);
        free(h);
    ROWS_END
    return 0;
}

/*
 * Fused bidirectional Mamba-1 scan: kernel/arm-scan-core/src/scalar.rs:114-201.
 * Pass A (discretize, exp, input projection) once per row into scratch, then
 * Pass B forward and backward over the shared products.  Bit-identical to two
 * oracle_m1_scan calls (forward, reverse) because the products are the same
 * values consumed in the same order.
 */
extern "C" int FN(oracle_m1_scan_bidir)(const oracle_m1_dims* dm, const T* u, const T* delta,
                             const T* a, const T* b, const T* c, const T* d_skip,
                             const T* z, const T* delta_bias, int delta_softplus,
                             T* out_fwd, T* out_bwd, T* last_fwd, T* last_bwd,
                             int nthreads) {
    if (!dm || !dm->batch || !dm->dim || !dm->len || !dm->state || !dm->groups ||
        dm->dim % dm->groups)
        return 2;
    if ((last_fwd == NULL) != (last_bwd == NULL)) return 2;
    const size_t dim = dm->dim, len = dm->len, state = dm->state;
    const size_t group_size = dim / dm->groups;
    ROWS_BEGIN(dm->batch * dim)
        T* abar = (T*)malloc(len * state * sizeof(T));
        T* bbar = (T*)malloc(len * state * sizeof(T));
        T* h = (T*)malloc(state * sizeof(T));
        for (size_t ch = r0; ch < r1; ++ch) {
            const size_t bi = ch / dim, d = ch % dim;
            const T* a_row = a + d * state;
            const T bias = delta_bias ? delta_bias[d] : (T)0;
            const size_t bc_base = (bi * dm->groups + d / group_size) * state * len;
            const size_t row = ch * len;
            for (size_t t = 0; t < len; ++t) {                /* Pass A, 160-172 */
                T dt = delta[row + t] + bias;
                if (delta_softplus) dt = FN(softplus)(dt);
                const T dt_u = dt * u[row + t];
                for (size_t n = 0; n < state; ++n) {
                    const size_t bc = bc_base + n * len + t;
                    abar[t * state + n] = EXP(dt * a_row[n]);
                    bbar[t * state + n] = dt_u * b[bc];
                }
            }
            for (int dir = 0; dir < 2; ++dir) {               /* Pass B, 177-199 */
                T* o = dir ? out_bwd : out_fwd;
                T* ls = dir ? last_bwd : last_fwd;
                for (size_t n = 0; n < state; ++n) h[n] = 0;
                for (size_t i = 0; i < len; ++i) {
                    const size_t t = dir ? len - 1 - i : i;
                    T y = 0;
                    for (size_t n = 0; n < state; ++n) {
                        const T nw = abar[t * state + n] * h[n] + bbar[t * state + n];
                        h[n] = nw;
                        y = y + c[bc_base + n * len + t] * nw;
                    }
                    if (d_skip) y = y + d_skip[d] * u[row + t];
                    if (z) y = y * FN(silu)(z[row + t]);
                    o[row + t] = y;
                }
                if (ls)
                    for (size_t n = 0; n < state; ++n) ls[ch * state + n] = h[n];
            }
        }
        free(abar); free(bbar); free(h);
    ROWS_END
    return 0;
}

/*
 * Mamba-3 gate terms for step t of a traversal (shared by SISO and MIMO):
 * kernel/arm-scan-core/src/mamba3/scalar.rs:160-186 and mimo.rs:143-158.
 * The trapezoid's second term reads the NEXT step in traversal order
 * (t+1 forward, t-1 backward); the last step of the traversal has none.
 */
static inline void FN(m3_gates)(const T* adt, const T* dt, const T* trap,
                                size_t gate_base, size_t len, size_t i,
                                int reverse, T* gamma, T* scale, T* alpha) {
    const size_t t = reverse ? len - 1 - i : i;
    const size_t g = gate_base + t;
    const T lam = FN(sigmoid)(trap[g]);
    *gamma = dt[g] * lam;
    T shifted = 0;
    if (i + 1 < len) {
        const size_t nx = reverse ? g - 1 : g + 1;
        shifted = dt[nx] * ((T)1 - FN(sigmoid)(trap[nx]));
    }
    *scale = *gamma + shifted;
    *alpha = EXP(adt[g]);
}

/*
 * Mamba-3 SISO scan: kernel/arm-scan-core/src/mamba3/scalar.rs:50-196.
 * Layouts (mamba3/mod.rs:44-56):
 *   q, k (batch, len, 1, dqk); v, z (batch, len, heads, dv)
 *   adt, dt, trap (batch, heads, len); cos, sin (batch, len, heads, dqk/2)
 *   q_bias, k_bias (heads, dqk); d_skip (heads,)
 *   out (batch, heads, len, dv)  -- head-major
 *   last_state (batch, heads, dv, dqk); last_bx (batch, heads, dqk)
 * RoPE is interleaved: lanes (2i, 2i+1) (scalar.rs:41-48).
 */
extern "C" int FN(oracle_m3_siso)(const oracle_m3_dims* dm, const T* q, const T* k,
                       const T* v, const T* adt, const T* dt, const T* trap,
                       const T* q_bias, const T* k_bias, const T* cosv,
                       const T* sinv, const T* d_skip, const T* z, int reverse,
                       T* out, T* last_state, T* last_bx, int nthreads) {
    if (!dm || !dm->batch || !dm->heads || !dm->dv || !dm->dqk || !dm->len ||
        dm->rank != 1 || (dm->dqk & 1))
        return 2;
    const size_t heads = dm->heads, dv = dm->dv, dqk = dm->dqk, len = dm->len;
    const size_t half = dqk / 2;
    ROWS_BEGIN(dm->batch * heads)
        T* S = (T*)malloc(dv * dqk * sizeof(T));
        T* qr = (T*)malloc(dqk * sizeof(T));
        T* kr = (T*)malloc(dqk * sizeof(T));
        T* bx = (T*)malloc(dqk * sizeof(T));
        for (size_t bh = r0; bh < r1; ++bh) {
            const size_t bi = bh / heads, h = bh % heads;
            const T* qb = q_bias + h * dqk;
            const T* kb = k_bias + h * dqk;
            const T dsk = d_skip ? d_skip[h] : (T)0;
            const size_t gate_base = (bi * heads + h) * len;
            for (size_t j = 0; j < dv * dqk; ++j) S[j] = 0;
            for (size_t j = 0; j < dqk; ++j) bx[j] = 0;
            for (size_t i = 0; i < len; ++i) {
                const size_t t = reverse ? len - 1 - i : i;
                T gamma, scale, alpha;
                FN(m3_gates)(adt, dt, trap, gate_base, len, i, reverse,
                             &gamma, &scale, &alpha);
                const size_t qk_off = (bi * len + t) * dqk;
                const size_t cs_off = ((bi * len + t) * heads + h) * half;
                for (size_t p = 0; p < half; ++p) {           /* rope, 41-48 */
                    const T cs = cosv[cs_off + p], sn = sinv[cs_off + p];
                    T x0 = q[qk_off + 2 * p] + qb[2 * p];
                    T x1 = q[qk_off + 2 * p + 1] + qb[2 * p + 1];
                    qr[2 * p] = x0 * cs - x1 * sn;
                    qr[2 * p + 1] = x0 * sn + x1 * cs;
                    x0 = k[qk_off + 2 * p] + kb[2 * p];
                    x1 = k[qk_off + 2 * p + 1] + kb[2 * p + 1];
                    kr[2 * p] = x0 * cs - x1 * sn;
                    kr[2 * p + 1] = x0 * sn + x1 * cs;
                }
                const size_t v_off = ((bi * len + t) * heads + h) * dv;
                T qk = 0;
                for (size_t j = 0; j < dqk; ++j) qk = qk + qr[j] * kr[j];
                const T diag = dsk + gamma * qk;
                T* o = out + (bh * len + t) * dv;
                for (size_t p = 0; p < dv; ++p) {             /* 224-235 */
                    T acc = 0;
                    for (size_t j = 0; j < dqk; ++j) acc = acc + qr[j] * S[p * dqk + j];
                    o[p] = alpha * acc + diag * v[v_off + p];
                }
                for (size_t p = 0; p < dv; ++p) {             /* 238-244 */
                    const T sv = scale * v[v_off + p];
                    for (size_t j = 0; j < dqk; ++j)
                        S[p * dqk + j] = alpha * S[p * dqk + j] + sv * kr[j];
                }
                for (size_t j = 0; j < dqk; ++j) bx[j] = scale * kr[j];
                if (z)
                    for (size_t p = 0; p < dv; ++p) o[p] = o[p] * FN(silu)(z[v_off + p]);
            }
            if (last_state)
                for (size_t j = 0; j < dv * dqk; ++j) last_state[bh * dv * dqk + j] = S[j];
            if (last_bx)
                for (size_t j = 0; j < dqk; ++j) last_bx[bh * dqk + j] = bx[j];
        }
        free(S); free(qr); free(kr); free(bx);
    ROWS_END
    return 0;
}

/*
 * Mamba-3 MIMO (rank r) scan: kernel/arm-scan-core/src/mamba3/mimo.rs:98-284.
 *   q, k (batch, len, rank, dqk); q_bias, k_bias (heads, rank, dqk)
 *   psi, zeta, phi (heads, rank, dv); cos, sin (batch, len, heads, dqk/2)
 * RoPE is split-halves over the first n_pairs lanes (mimo.rs:83-96), where
 * n_pairs = min(cos row length, dqk/2) = `pairs` here.
 * last_state (batch, heads, dv, dqk) is written when non-null; the reference
 * rejects it for MIMO at its C boundary but the state itself is well defined
 * (mimo.rs:278-280 copies it out).
 */
extern "C" int FN(oracle_m3_mimo)(const oracle_m3_dims* dm, const T* q, const T* k,
                       const T* v, const T* adt, const T* dt, const T* trap,
                       const T* q_bias, const T* k_bias, const T* cosv,
                       const T* sinv, const T* d_skip, const T* z,
                       const T* psi, const T* zeta, const T* phi, size_t pairs,
                       int reverse, T* out, T* last_state, int nthreads) {
    if (!dm || !dm->batch || !dm->heads || !dm->dv || !dm->dqk || !dm->len ||
        !dm->rank || (dm->dqk & 1))
        return 2;
    const size_t heads = dm->heads, dv = dm->dv, dqk = dm->dqk, len = dm->len;
    const size_t R = dm->rank, half = dqk / 2;
    if (pairs > half) pairs = half;
    ROWS_BEGIN(dm->batch * heads)
        T* S = (T*)malloc(dv * dqk * sizeof(T));
        T* qr = (T*)malloc(R * dqk * sizeof(T));
        T* kr = (T*)malloc(R * dqk * sizeof(T));
        T* x = (T*)malloc(R * dv * sizeof(T));
        T* acc = (T*)malloc(R * dv * sizeof(T));
        T* gram = (T*)malloc(R * R * sizeof(T));
        for (size_t bh = r0; bh < r1; ++bh) {
            const size_t bi = bh / heads, h = bh % heads;
            const size_t bias_base = h * R * dqk, proj_base = h * R * dv;
            const T dsk = d_skip ? d_skip[h] : (T)0;
            const size_t gate_base = (bi * heads + h) * len;
            for (size_t j = 0; j < dv * dqk; ++j) S[j] = 0;
            for (size_t i = 0; i < len; ++i) {
                const size_t t = reverse ? len - 1 - i : i;
                T gamma, scale, alpha;
                FN(m3_gates)(adt, dt, trap, gate_base, len, i, reverse,
                             &gamma, &scale, &alpha);
                const size_t cs_off = ((bi * len + t) * heads + h) * half;
                const size_t qk_off = (bi * len + t) * R * dqk;
                for (size_t r = 0; r < R; ++r) {              /* 164-181 */
                    T* qd = qr + r * dqk; T* kd = kr + r * dqk;
                    for (size_t j = 0; j < dqk; ++j) {
                        qd[j] = q[qk_off + r * dqk + j] + q_bias[bias_base + r * dqk + j];
                        kd[j] = k[qk_off + r * dqk + j] + k_bias[bias_base + r * dqk + j];
                    }
                    for (size_t p = 0; p < pairs; ++p) {
                        const T cs = cosv[cs_off + p], sn = sinv[cs_off + p];
                        T a0 = qd[p], a1 = qd[half + p];
                        qd[p] = a0 * cs - a1 * sn; qd[half + p] = a0 * sn + a1 * cs;
                        a0 = kd[p]; a1 = kd[half + p];
                        kd[p] = a0 * cs - a1 * sn; kd[half + p] = a0 * sn + a1 * cs;
                    }
                }
                const size_t v_off = ((bi * len + t) * heads + h) * dv;
                for (size_t r = 0; r < R; ++r)                /* 188-196 */
                    for (size_t p = 0; p < dv; ++p)
                        x[r * dv + p] = psi[proj_base + r * dv + p] * v[v_off + p];
                for (size_t ra = 0; ra < R; ++ra)             /* 199-206 */
                    for (size_t rb = 0; rb < R; ++rb) {
                        T s = 0;
                        for (size_t j = 0; j < dqk; ++j) s = s + qr[ra * dqk + j] * kr[rb * dqk + j];
                        gram[ra * R + rb] = s;
                    }
                for (size_t r = 0; r < R; ++r)                /* 209-231 */
                    for (size_t p = 0; p < dv; ++p) {
                        T s = 0;
                        for (size_t j = 0; j < dqk; ++j) s = s + qr[r * dqk + j] * S[p * dqk + j];
                        T dg = 0;
                        for (size_t rb = 0; rb < R; ++rb) dg = dg + gram[r * R + rb] * x[rb * dv + p];
                        acc[r * dv + p] = alpha * s + gamma * dg + dsk * x[r * dv + p];
                    }
                for (size_t p = 0; p < dv; ++p)               /* 234-242 */
                    for (size_t j = 0; j < dqk; ++j) {
                        T upd = 0;
                        for (size_t r = 0; r < R; ++r) upd = upd + x[r * dv + p] * kr[r * dqk + j];
                        S[p * dqk + j] = alpha * S[p * dqk + j] + scale * upd;
                    }
                T* o = out + (bh * len + t) * dv;             /* 250-273 */
                for (size_t p = 0; p < dv; ++p) o[p] = 0;
                for (size_t r = 0; r < R; ++r)
                    for (size_t p = 0; p < dv; ++p) {
                        const T ph = phi[proj_base + r * dv + p];
                        if (z) {
                            const T g = FN(silu)(z[v_off + p] * zeta[proj_base + r * dv + p]);
                            o[p] = o[p] + ph * g * acc[r * dv + p];
                        } else {
                            o[p] = o[p] + ph * acc[r * dv + p];
                        }
                    }
            }
            if (last_state)
                for (size_t j = 0; j < dv * dqk; ++j) last_state[bh * dv * dqk + j] = S[j];
        }
        free(S); free(qr); free(kr); free(x); free(acc); free(gram);
    ROWS_END
    return 0;
}

/*
 * Mamba-3 MIMO with the input given per rank (the configuration whose state
 * recurrence is written out in terms of X, B, C):
 *   h_t = alpha_t h_{t-1} + beta_t X_{t-1} B_{t-1}^T + gamma_t X_t B_t^T
 *   Y_t = h_t C_t (+ D X_t)
 * per (batch, head), h of shape (dv, dqk), X_t of shape (dv, rank),
 * B_t, C_t of shape (dqk, rank).  The gates are the SISO/MIMO ones of
 * tests/reference/mamba3_ref.py:27-39 (FN(m3_gates) above):
 *   alpha_t = exp(adt_t), gamma_t = dt_t sigmoid(trap_t),
 *   beta_t  = alpha_t dt_t (1 - sigmoid(trap_t))  -- the trapezoid's share
 * of the previous step, decayed by this step's alpha (mamba3_ref.py:27-39);
 * "previous" is t-1 forward and t+1 under reverse; the first step of a
 * traversal has no previous term.  B and C are RoPE-rotated split-halves
 * over the first `pairs` lanes (mamba3_ref.py:285-298) with the step's
 * cos/sin, as in the MIMO op.  This is the op of mamba3_ref.py:305-411 with
 * x_r given directly (replacing the psi projection at :384) and the per-rank
 * outputs returned without the zeta gate and phi reduction (:405-411).
 * Layouts: x, out (batch, len, heads, dv, rank); b, c (batch, len, dqk, rank);
 * adt, dt, trap (batch, heads, len); cos, sin (batch, len, heads, dqk/2);
 * d_skip (heads) nullable; last_state (batch, heads, dv, dqk) = h after the
 * last step.
 */
extern "C" int FN(oracle_m3_mimo_x)(const oracle_m3_dims* dm, const T* x, const T* bm,
                       const T* cm, const T* adt, const T* dt, const T* trap,
                       const T* cosv, const T* sinv, size_t pairs, const T* d_skip,
                       int reverse, T* out, T* last_state, int nthreads) {
    if (!dm || !dm->batch || !dm->heads || !dm->dv || !dm->dqk || !dm->len ||
        !dm->rank || (dm->dqk & 1))
        return 2;
    const size_t heads = dm->heads, P = dm->dv, N = dm->dqk, len = dm->len;
    const size_t R = dm->rank, half = N / 2;
    if (pairs > half) pairs = half;
    ROWS_BEGIN(dm->batch * heads)
        T* h = (T*)malloc(P * N * sizeof(T));
        T* br = (T*)malloc(N * R * sizeof(T));     /* this step's rotated B [n][r] */
        T* bp = (T*)malloc(N * R * sizeof(T));     /* previous step's rotated B */
        T* cr = (T*)malloc(N * R * sizeof(T));
        T* xp = (T*)malloc(P * R * sizeof(T));     /* previous step's X */
        for (size_t bh = r0; bh < r1; ++bh) {
            const size_t bi = bh / heads, hd = bh % heads;
            const size_t gate_base = (bi * heads + hd) * len;
            const T dsk = d_skip ? d_skip[hd] : (T)0;
            for (size_t j = 0; j < P * N; ++j) h[j] = 0;
            for (size_t i = 0; i < len; ++i) {
                const size_t t = reverse ? len - 1 - i : i;
                const size_t g = gate_base + t;
                const T lam = FN(sigmoid)(trap[g]);
                const T alpha = EXP(adt[g]);
                const T gamma = dt[g] * lam;
                const T beta = alpha * dt[g] * ((T)1 - lam);
                const size_t bc_off = (bi * len + t) * N * R;
                const size_t cs_off = ((bi * len + t) * heads + hd) * half;
                for (size_t n = 0; n < N * R; ++n) { br[n] = bm[bc_off + n]; cr[n] = cm[bc_off + n]; }
                for (size_t pr = 0; pr < pairs; ++pr) {
                    const T cs = cosv[cs_off + pr], sn = sinv[cs_off + pr];
                    for (size_t r = 0; r < R; ++r) {
                        T a0 = br[pr * R + r], a1 = br[(half + pr) * R + r];
                        br[pr * R + r] = a0 * cs - a1 * sn; br[(half + pr) * R + r] = a0 * sn + a1 * cs;
                        a0 = cr[pr * R + r]; a1 = cr[(half + pr) * R + r];
                        cr[pr * R + r] = a0 * cs - a1 * sn; cr[(half + pr) * R + r] = a0 * sn + a1 * cs;
                    }
                }
                const T* xt = x + ((bi * len + t) * heads + hd) * P * R;
                for (size_t p = 0; p < P; ++p)
                    for (size_t n = 0; n < N; ++n) {
                        T cur = 0, prev = 0;
                        for (size_t r = 0; r < R; ++r) {
                            cur = cur + xt[p * R + r] * br[n * R + r];
                            if (i > 0) prev = prev + xp[p * R + r] * bp[n * R + r];
                        }
                        h[p * N + n] = alpha * h[p * N + n] + beta * prev + gamma * cur;
                    }
                T* o = out + ((bi * len + t) * heads + hd) * P * R;
                for (size_t p = 0; p < P; ++p)
                    for (size_t r = 0; r < R; ++r) {
                        T s = 0;
                        for (size_t n = 0; n < N; ++n) s = s + h[p * N + n] * cr[n * R + r];
                        o[p * R + r] = s + dsk * xt[p * R + r];
                    }
                for (size_t j = 0; j < P * R; ++j) xp[j] = xt[j];
                for (size_t n = 0; n < N * R; ++n) bp[n] = br[n];
            }
            if (last_state)
                for (size_t j = 0; j < P * N; ++j) last_state[bh * P * N + j] = h[j];
        }
        free(h); free(br); free(bp); free(cr); free(xp);
    ROWS_END
    return 0;
}
