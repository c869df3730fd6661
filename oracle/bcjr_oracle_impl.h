/*
 * Body of the CPU oracle, included twice by bcjr_oracle.c with
 *   REAL = double, SUFFIX(name) = name##_f64   (error attribution)
 *   REAL = float,  SUFFIX(name) = name##_f32   (same operation order as the
 *                                               reference's fp32 torch path)
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain restatement of the reference's
 * eager BCJR algorithm (src/bcjr/forward_backward.py) and of its analytic
 * backward (src/bcjr/bcjr_monolithic.py).  Nothing in the product calls it.
 *
 * Every array is materialised exactly as the reference does:
 *   log_local (N,S), log_alpha (N,S), log_beta (N,S), P computed on the fly,
 *   and the two adjoint sweeps of the monolithic backward.
 */

/* logsumexp with the max shift used by torch.logsumexp
 * (forward_backward.py:111, :119, :220). */
static REAL SUFFIX(lse)(const REAL *x, long n) {
    REAL m = x[0];
    for (long i = 1; i < n; ++i) if (x[i] > m) m = x[i];
    REAL s = 0;
    for (long i = 0; i < n; ++i) s += EXP(x[i] - m);
    return m + LOG(s);
}

/*
 * One sequence: forward (soft, logZ) and, when grad_soft != NULL, the
 * gradient d_seq.  seq: (N,V), cb: (S,V), soft: (N,V), d_seq: (N,V).
 * Scratch is allocated here (4 * N * S reals at most).
 * Returns 0 on success, -1 on allocation failure.
 */
static int SUFFIX(one_sequence)(const REAL *seq, const REAL *cb, REAL T,
                               int N, int L, int b, int V,
                               REAL *soft, REAL *logZ_out,
                               const REAL *grad_soft, REAL *d_seq,
                               int inner_parallel) {
    const long S = 1L << L;
    const int NB = 1 << b;                 /* predecessors per state */
    const long mask = S - 1;
    REAL *ll = (REAL *)malloc(sizeof(REAL) * N * S);
    REAL *la = (REAL *)malloc(sizeof(REAL) * N * S);
    REAL *lb = (REAL *)malloc(sizeof(REAL) * N * S);
    REAL *dla = grad_soft ? (REAL *)malloc(sizeof(REAL) * N * S) : NULL;
    REAL *cb_sq = (REAL *)malloc(sizeof(REAL) * S);
    if (!ll || !la || !lb || !cb_sq || (grad_soft && !dla)) {
        free(ll); free(la); free(lb); free(dla); free(cb_sq);
        return -1;
    }

    /* _local_log_prob, forward_backward.py:89-103:
     *   -( |cb|^2 - 2 <cb, w> + |w|^2 ) / T   (same expansion, same order) */
    for (long s = 0; s < S; ++s) {
        REAL a = 0;
        for (int v = 0; v < V; ++v) a += cb[s * V + v] * cb[s * V + v];
        cb_sq[s] = a;
    }
    for (int t = 0; t < N; ++t) {
        REAL wsq = 0;
        for (int v = 0; v < V; ++v) wsq += seq[t * V + v] * seq[t * V + v];
        for (long s = 0; s < S; ++s) {
            REAL dot = 0;
            for (int v = 0; v < V; ++v) dot += seq[t * V + v] * cb[s * V + v];
            REAL cost = cb_sq[s] - (REAL)2.0 * dot + wsq;
            ll[(long)t * S + s] = -cost / T;
        }
    }

    /* _forward_log_alpha, forward_backward.py:122-154, with the step of
     * :106-112.  preds[s,p] = (p << (L-b)) | (s >> b)   (:78-80).
     * log_alpha_{-1} = 0. */
    for (int t = 0; t < N; ++t) {
        for (long s = 0; s < S; ++s) {
            REAL g[16];
            for (int p = 0; p < NB; ++p) {
                long q = ((long)p << (L - b)) | (s >> b);
                g[p] = t ? la[(long)(t - 1) * S + q] : (REAL)0;
            }
            la[(long)t * S + s] = ll[(long)t * S + s] + SUFFIX(lse)(g, NB);
        }
    }

    /* _backward_log_beta, forward_backward.py:157-187, step :115-119.
     * succs[s,c] = ((s << b) | c) & mask   (:82-84).  log_beta_{N-1} = 0. */
    for (long s = 0; s < S; ++s) lb[(long)(N - 1) * S + s] = 0;
    for (int t = N - 2; t >= 0; --t) {
        for (long s = 0; s < S; ++s) {
            REAL g[16];
            for (int c = 0; c < NB; ++c) {
                long q = ((s << b) | c) & mask;
                g[c] = ll[(long)(t + 1) * S + q] + lb[(long)(t + 1) * S + q];
            }
            lb[(long)t * S + s] = SUFFIX(lse)(g, NB);
        }
    }

    /* log_Z = logsumexp(log_alpha[N-1]), forward_backward.py:220 */
    const REAL logZ = SUFFIX(lse)(la + (long)(N - 1) * S, S);
    *logZ_out = logZ;

    /* P = exp(alpha + beta - logZ); soft = P @ cb   (:223-228) */
    for (int t = 0; t < N; ++t) {
        for (int v = 0; v < V; ++v) {
            REAL acc = 0;
            for (long s = 0; s < S; ++s) {
                REAL P = EXP(la[(long)t * S + s] + lb[(long)t * S + s] - logZ);
                acc += P * cb[s * V + v];
            }
            soft[t * V + v] = acc;
        }
    }

    if (grad_soft) {
        /* BcjrForwardBackwardMonolithic.backward, bcjr_monolithic.py:191-243 */
        /* d_log_P[t,s] = P[t,s] * <grad_soft[t], cb[s]>  (:198-201);
         * d_log_Z = -sum d_log_P  (:207) */
        REAL dlogZ = 0;
        for (int t = 0; t < N; ++t)
            for (long s = 0; s < S; ++s) {
                REAL P = EXP(la[(long)t * S + s] + lb[(long)t * S + s] - logZ);
                REAL dP = 0;
                for (int v = 0; v < V; ++v) dP += grad_soft[t * V + v] * cb[s * V + v];
                dla[(long)t * S + s] = P * dP;      /* d_log_alpha = d_log_P */
                dlogZ -= P * dP;
            }
        /* d_log_alpha[N-1] += softmax(alpha[N-1]) * d_log_Z  (:211-216) */
        for (long s = 0; s < S; ++s)
            dla[(long)(N - 1) * S + s] += EXP(la[(long)(N - 1) * S + s] - logZ) * dlogZ;

        /* _backward_log_alpha (:104-127): reverse sweep.  dla[t] becomes the
         * alpha-part of d_log_local[t] in place. */
        REAL *gprev = (REAL *)calloc(S, sizeof(REAL));
        for (int t = N - 1; t >= 1; --t) {
            memset(gprev, 0, sizeof(REAL) * S);
            const REAL *ap = la + (long)(t - 1) * S;
            const REAL *gn = dla + (long)t * S;          /* total adjoint of alpha_t */
            /* softmax of the predecessor group is shared by the 2^b states
             * with the same s >> b; scatter exactly as the atomic kernel. */
            for (long s = 0; s < S; ++s) {
                REAL g[16];
                for (int p = 0; p < NB; ++p) g[p] = ap[((long)p << (L - b)) | (s >> b)];
                REAL m = g[0];
                for (int p = 1; p < NB; ++p) if (g[p] > m) m = g[p];
                REAL e[16], se = 0;
                for (int p = 0; p < NB; ++p) { e[p] = EXP(g[p] - m); se += e[p]; }
                for (int p = 0; p < NB; ++p)
                    gprev[((long)p << (L - b)) | (s >> b)] += gn[s] * (e[p] / se);
            }
            for (long s = 0; s < S; ++s) dla[(long)(t - 1) * S + s] += gprev[s];
        }

        /* _backward_log_beta (:130-154): forward sweep; dlb[t+1] accumulates
         * into dla (d_log_local = alpha part + beta part, :226). */
        REAL *gbeta = (REAL *)malloc(sizeof(REAL) * S);
        REAL *gx = gprev;
        /* grad_beta_prev = d_log_beta[0] = d_log_P[0] */
        for (long s = 0; s < S; ++s) {
            REAL P = EXP(la[s] + lb[s] - logZ);
            REAL dP = 0;
            for (int v = 0; v < V; ++v) dP += grad_soft[v] * cb[s * V + v];
            gbeta[s] = P * dP;
        }
        for (int t = 0; t < N - 1; ++t) {
            memset(gx, 0, sizeof(REAL) * S);
            for (long s = 0; s < S; ++s) {
                REAL x[16];
                for (int c = 0; c < NB; ++c) {
                    long q = ((s << b) | c) & mask;
                    x[c] = ll[(long)(t + 1) * S + q] + lb[(long)(t + 1) * S + q];
                }
                REAL m = x[0];
                for (int c = 1; c < NB; ++c) if (x[c] > m) m = x[c];
                REAL e[16], se = 0;
                for (int c = 0; c < NB; ++c) { e[c] = EXP(x[c] - m); se += e[c]; }
                for (int c = 0; c < NB; ++c)
                    gx[((s << b) | c) & mask] += gbeta[s] * (e[c] / se);
            }
            for (long s = 0; s < S; ++s) {
                REAL P = EXP(la[(long)(t + 1) * S + s] + lb[(long)(t + 1) * S + s] - logZ);
                REAL dP = 0;
                for (int v = 0; v < V; ++v) dP += grad_soft[(t + 1) * V + v] * cb[s * V + v];
                dla[(long)(t + 1) * S + s] += gx[s];
                gbeta[s] = P * dP + gx[s];
            }
        }
        free(gbeta);
        free(gprev);

        /* d_w = (2/T) d_ll @ cb - (2/T) w * sum_s d_ll   (:232-239) */
        const REAL invT = (REAL)1.0 / T;
        for (int t = 0; t < N; ++t) {
            REAL dsum = 0;
            for (long s = 0; s < S; ++s) dsum += dla[(long)t * S + s];
            for (int v = 0; v < V; ++v) {
                REAL acc = 0;
                for (long s = 0; s < S; ++s) acc += dla[(long)t * S + s] * cb[s * V + v];
                d_seq[t * V + v] = ((REAL)2.0 * invT) * acc
                                 + ((REAL)-2.0 * invT) * seq[t * V + v] * dsum;
            }
        }
    }
    free(ll); free(la); free(lb); free(dla); free(cb_sq);
    return 0;
}

/* Work queue over sequences: each worker thread takes the next sequence. */
typedef struct {
    const REAL *seq, *cb; REAL T; int N, L, b, V;
    REAL *soft, *logZ; const REAL *grad_soft; REAL *d_seq;
    int B, next, err; pthread_mutex_t lock;
} SUFFIX(job_t);

static void *SUFFIX(worker)(void *arg) {
    SUFFIX(job_t) *j = (SUFFIX(job_t) *)arg;
    for (;;) {
        pthread_mutex_lock(&j->lock);
        int i = j->next++;
        pthread_mutex_unlock(&j->lock);
        if (i >= j->B) break;
        long o = (long)i * j->N * j->V;
        int e = SUFFIX(one_sequence)(j->seq + o, j->cb, j->T, j->N, j->L, j->b, j->V,
                                     j->soft + o, j->logZ + i,
                                     j->grad_soft ? j->grad_soft + o : NULL,
                                     j->d_seq ? j->d_seq + o : NULL, 0);
        if (e) { pthread_mutex_lock(&j->lock); j->err = 1; pthread_mutex_unlock(&j->lock); }
    }
    return NULL;
}

/* Batch entry: B independent sequences, one worker thread per sequence at a
 * time (nthreads workers). */
int SUFFIX(bcjr_oracle)(const REAL *seq, const REAL *cb, REAL T,
                        int B, int N, int L, int k, int V,
                        REAL *soft, REAL *logZ,
                        const REAL *grad_soft, REAL *d_seq, int nthreads) {
    const int b = k * V;
    if (B < 0 || N < 1 || V < 1 || b < 1 || b > 4 || L < b || L > 20) return -2;
    SUFFIX(job_t) job;
    memset(&job, 0, sizeof(job));
    job.seq = seq; job.cb = cb; job.T = T; job.N = N; job.L = L; job.b = b; job.V = V;
    job.soft = soft; job.logZ = logZ; job.grad_soft = grad_soft; job.d_seq = d_seq;
    job.B = B;
    pthread_mutex_init(&job.lock, NULL);
    run_parallel(SUFFIX(worker), &job, nthreads > 0 ? nthreads : 1, B);
    pthread_mutex_destroy(&job.lock);
    return job.err ? -1 : 0;
}
