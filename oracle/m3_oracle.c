/* m3_oracle.c -- TEST INFRASTRUCTURE (oracle). Not part of the product.
 *
 * A plain-C restatement of the reference's IVF search path and of the k-means /
 * split procedure this project specifies (the reference has none).  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it, and only as
 * the checker.  The product path never calls it.
 *
 * Arithmetic follows the reference exactly: fp32, one rounding per multiply, add
 * and subtract, summed in index order (AgentMemory/M3/src/base.cpp:12-41; the
 * reference is built without -march, so x86-64 GCC never contracts to FMA).  This
 * file must therefore be compiled with -ffp-contract=off (oracle/Makefile does).
 *
 * The restatement is pinned against the reference core itself (liboracle_ref.so,
 * built from the reference sources by oracle/Makefile) and against the golden
 * fixtures under tests/golden/ that were produced by that same reference core.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORC_L2 = 0, ORC_IP = 1, ORC_COSINE = 2 };

/* unified_score: AgentMemory/M3/include/base.h:22-31, kernels base.cpp:12-41.
 * Smaller is better for every metric. */
float orc_score(const float* a, const float* b, int d, int metric, int normalized) {
    if (metric == ORC_L2) { /* base.cpp:12-20 */
        float s = 0.f;
        for (int i = 0; i < d; ++i) {
            float df = a[i] - b[i];
            s += df * df;
        }
        return s;
    }
    if (metric == ORC_IP || normalized) { /* base.cpp:22-29 */
        float s = 0.f;
        for (int i = 0; i < d; ++i) s += a[i] * b[i];
        return metric == ORC_IP ? -s : 1.f - s;
    }
    /* COSINE, not normalized: base.cpp:31-41 */
    float dot = 0.f, na = 0.f, nb = 0.f;
    for (int i = 0; i < d; ++i) {
        dot += a[i] * b[i];
        na += a[i] * a[i];
        nb += b[i] * b[i];
    }
    if (na == 0.f || nb == 0.f) return 1.f;
    return 1.f - dot / sqrtf(na * nb);
}

typedef struct {
    float s;
    int32_t c;
} orc_sc;

static int orc_sc_cmp(const void* x, const void* y) {
    const orc_sc* a = (const orc_sc*)x;
    const orc_sc* b = (const orc_sc*)y;
    if (a->s < b->s) return -1;
    if (b->s < a->s) return 1;
    return (a->c > b->c) - (a->c < b->c);
}

/* select_nprobe_for_query: AgentMemory/M3/src/m3_index.cpp:492-523.
 * The reference picks the nprobe smallest with nth_element + sort (ties in an
 * unspecified order); this restatement breaks exact ties by the lower cluster id.
 * Returns the number written (min(nprobe, nlist)); out is ascending by score. */
int orc_select_nprobe(const float* q, const float* C, int nlist, int d, int metric,
                      int normalized, int nprobe, int32_t* out) {
    if (nlist <= 0 || nprobe <= 0) return 0;
    orc_sc* t = (orc_sc*)malloc(sizeof(orc_sc) * (size_t)nlist);
    for (int c = 0; c < nlist; ++c) {
        t[c].s = orc_score(q, C + (size_t)c * d, d, metric, normalized);
        t[c].c = c;
    }
    qsort(t, (size_t)nlist, sizeof(orc_sc), orc_sc_cmp);
    int m = nprobe < nlist ? nprobe : nlist;
    for (int i = 0; i < m; ++i) out[i] = t[i].c;
    free(t);
    return m;
}

/* nearest_clusters: AgentMemory/M3/src/m3_index.cpp:243-264.  Strict '<', so the
 * lowest cluster id wins an exact tie; -1 when nlist == 0 (or every score NaN). */
void orc_nearest_clusters(const float* X, int64_t n, const float* C, int nlist, int d,
                          int metric, int normalized, int32_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        float best = INFINITY;
        int32_t bid = -1;
        for (int c = 0; c < nlist; ++c) {
            float s = orc_score(X + (size_t)i * d, C + (size_t)c * d, d, metric, normalized);
            if (s < best) {
                best = s;
                bid = c;
            }
        }
        out[i] = bid;
    }
}

/* Cluster::search_into: AgentMemory/M3/src/cluster.cpp:229-274.  Unsorted k-slot
 * buffer; a row replaces the current worst slot (first maximum) on a strict '<'. */
static void orc_search_into(const float* q, int d, int metric, int normalized, const float* vecs,
                            const int64_t* ids, const uint8_t* alive, int64_t n, int k,
                            int64_t* top_ids, float* top_s) {
    if (n == 0) return;
    int wi = 0;
    for (int i = 1; i < k; ++i)
        if (top_s[i] > top_s[wi]) wi = i;
    float ws = top_s[wi];
    for (int64_t r = 0; r < n; ++r) {
        if (alive && !alive[r]) continue;
        float s = orc_score(q, vecs + (size_t)r * d, d, metric, normalized);
        if (s < ws) {
            top_ids[wi] = ids[r];
            top_s[wi] = s;
            wi = 0;
            for (int i = 1; i < k; ++i)
                if (top_s[i] > top_s[wi]) wi = i;
            ws = top_s[wi];
        }
    }
}

typedef struct {
    float s;
    int32_t slot;
} orc_slot;

static int orc_slot_cmp(const void* x, const void* y) {
    const orc_slot* a = (const orc_slot*)x;
    const orc_slot* b = (const orc_slot*)y;
    if (a->s < b->s) return -1;
    if (b->s < a->s) return 1;
    return (a->slot > b->slot) - (a->slot < b->slot);
}

/* Finalise one query's buffer: drop -1 slots, sort ascending by score
 * (AgentMemory/M3/src/m3_index.cpp:444-475).  Pads the row with -1 / +inf. */
static int orc_finish(int k, const int64_t* top_ids, const float* top_s, int64_t* out_ids,
                      float* out_s) {
    orc_slot* t = (orc_slot*)malloc(sizeof(orc_slot) * (size_t)k);
    int m = 0;
    for (int i = 0; i < k; ++i)
        if (top_ids[i] != -1) {
            t[m].s = top_s[i];
            t[m].slot = i;
            ++m;
        }
    qsort(t, (size_t)m, sizeof(orc_slot), orc_slot_cmp);
    for (int i = 0; i < k; ++i) {
        out_ids[i] = i < m ? top_ids[t[i].slot] : -1;
        out_s[i] = i < m ? top_s[t[i].slot] : INFINITY;
    }
    free(t);
    return m;
}

/* search_on: AgentMemory/M3/src/m3_index.cpp:314-366 (explicit cluster list). */
int orc_search_on(const float* Q, int64_t nq, int d, int metric, int normalized,
                  const int64_t* list_off, int nlist, const float* vecs, const int64_t* ids,
                  const uint8_t* alive, const int32_t* cids, int ncids, int k, int64_t* out_ids,
                  float* out_s, int32_t* out_counts) {
    if (k <= 0) return 0;
    int64_t* ti = (int64_t*)malloc(sizeof(int64_t) * (size_t)k);
    float* ts = (float*)malloc(sizeof(float) * (size_t)k);
    for (int64_t qi = 0; qi < nq; ++qi) {
        const float* q = Q + (size_t)qi * d;
        for (int i = 0; i < k; ++i) {
            ti[i] = -1;
            ts[i] = INFINITY;
        }
        for (int j = 0; j < ncids; ++j) {
            int c = cids[j];
            if (c < 0 || c >= nlist) continue;
            int64_t b = list_off[c], e = list_off[c + 1];
            orc_search_into(q, d, metric, normalized, vecs + (size_t)b * d, ids + b,
                            alive ? alive + b : NULL, e - b, k, ti, ts);
        }
        out_counts[qi] = orc_finish(k, ti, ts, out_ids + (size_t)qi * k, out_s + (size_t)qi * k);
    }
    free(ti);
    free(ts);
    return 0;
}

/* search_nprobe: AgentMemory/M3/src/m3_index.cpp:368-483.  nprobe <= 0 means every
 * list (:387); nprobe is clamped to nlist (:388).  Lists are given as CSR:
 * rows list_off[c] .. list_off[c+1]-1 of vecs/ids/alive belong to cluster c, in
 * the cluster's row order.  Also writes the chosen probes (ascending score,
 * padded with -1) when probes != NULL. */
int orc_search_nprobe(const float* Q, int64_t nq, int d, int metric, int normalized,
                      const float* C, int nlist, const int64_t* list_off, const float* vecs,
                      const int64_t* ids, const uint8_t* alive, int k, int nprobe,
                      int64_t* out_ids, float* out_s, int32_t* out_counts, int32_t* probes) {
    if (k <= 0 || nlist <= 0) {
        for (int64_t i = 0; i < nq; ++i) out_counts[i] = 0;
        return 0;
    }
    if (nprobe <= 0) nprobe = nlist;
    int p = nprobe < nlist ? nprobe : nlist;
    int32_t* ch = (int32_t*)malloc(sizeof(int32_t) * (size_t)p);
    for (int64_t qi = 0; qi < nq; ++qi) {
        const float* q = Q + (size_t)qi * d;
        int m = orc_select_nprobe(q, C, nlist, d, metric, normalized, p, ch);
        if (probes)
            for (int j = 0; j < p; ++j) probes[(size_t)qi * p + j] = j < m ? ch[j] : -1;
        orc_search_on(q, 1, d, metric, normalized, list_off, nlist, vecs, ids, alive, ch, m, k,
                      out_ids + (size_t)qi * k, out_s + (size_t)qi * k, out_counts + qi);
    }
    free(ch);
    return 0;
}

/* ---------------- k-means and split (no reference counterpart) ----------------
 *
 * The reference never trains centroids (AgentMemory/M3/src/m3_index.cpp:304-311 is
 * a TODO).  This is the procedure the product specifies, restated here:
 *   init   : nlist distinct rows chosen by orc_sample_rows(seed)
 *   E-step : nearest_clusters above (the reference's own rule, strict '<')
 *   M-step : per cluster, the fp64 sum of its rows in ascending row order,
 *            divided by the count in fp64, rounded to fp32; an empty cluster
 *            keeps its previous centroid.  The nearest running-mean semantics in
 *            the reference are AgentMemory/M3/src/m3_multi_level.cpp:131-148.
 *   final  : assignment against the last centroids. */

static uint64_t orc_splitmix64(uint64_t* st) {
    uint64_t z = (*st += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* m distinct indices of [0, n) by a seeded partial Fisher-Yates shuffle:
 * for i < m: j = i + splitmix64() % (n - i); swap(perm[i], perm[j]). */
int orc_sample_rows(uint64_t seed, int64_t n, int64_t m, int64_t* out) {
    if (m > n || m < 0) return -1;
    int64_t* perm = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    for (int64_t i = 0; i < n; ++i) perm[i] = i;
    uint64_t st = seed;
    for (int64_t i = 0; i < m; ++i) {
        int64_t j = i + (int64_t)(orc_splitmix64(&st) % (uint64_t)(n - i));
        int64_t t = perm[i];
        perm[i] = perm[j];
        perm[j] = t;
        out[i] = perm[i];
    }
    free(perm);
    return 0;
}

void orc_kmeans_update(const float* X, int64_t n, int d, const int32_t* assign, int nlist,
                       float* C) {
    double* acc = (double*)calloc((size_t)nlist * d, sizeof(double));
    int64_t* cnt = (int64_t*)calloc((size_t)nlist, sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) {
        int a = assign[i];
        if (a < 0 || a >= nlist) continue;
        double* s = acc + (size_t)a * d;
        const float* x = X + (size_t)i * d;
        for (int j = 0; j < d; ++j) s[j] += (double)x[j];
        cnt[a]++;
    }
    for (int c = 0; c < nlist; ++c) {
        if (cnt[c] == 0) continue;
        for (int j = 0; j < d; ++j)
            C[(size_t)c * d + j] = (float)(acc[(size_t)c * d + j] / (double)cnt[c]);
    }
    free(acc);
    free(cnt);
}

int orc_kmeans_train(const float* X, int64_t n, int d, int metric, int normalized, int nlist,
                     int niter, uint64_t seed, float* C, int32_t* assign) {
    if (nlist <= 0 || nlist > n) return -1;
    int64_t* init = (int64_t*)malloc(sizeof(int64_t) * (size_t)nlist);
    orc_sample_rows(seed, n, nlist, init);
    for (int c = 0; c < nlist; ++c)
        memcpy(C + (size_t)c * d, X + (size_t)init[c] * d, sizeof(float) * (size_t)d);
    free(init);
    for (int it = 0; it < niter; ++it) {
        orc_nearest_clusters(X, n, C, nlist, d, metric, normalized, assign);
        orc_kmeans_update(X, n, d, assign, nlist, C);
    }
    orc_nearest_clusters(X, n, C, nlist, d, metric, normalized, assign);
    return 0;
}

/* The GEMM estimate of one unified score and its error bound (see below). */
static inline void orc_interval(int metric, float s, double xi, double ci, double g, double g3,
                                double* est, double* e) {
    const double u = 1.0 / 16777216.0;
    const double e0 = 2.0 * g * xi * ci;
    if (metric == ORC_IP) {
        *est = -(double)s;
        *e = e0;
    } else if (metric == ORC_COSINE) {
        *est = 1.0 - (double)s;
        *e = e0 + 1.01 * u * (fabs(*est) + e0);
    } else {
        *est = xi * xi + ci * ci - 2.0 * (double)s;
        *e = 2.0 * e0 + g3 * (fabs(*est) + 2.0 * e0) + 4.0 * u * u * (xi * xi + ci * ci);
    }
}

/* The nearest_clusters rule above (strict '<', lowest id on exact ties) for large
 * inputs, given S[n, nlist] = X C^T from any fp32 GEMM (BLAS: any summation order,
 * FMA or not).  For every row the GEMM's estimate of each unified score is within
 * a rigorous bound e_c of the exact score; only the centroids whose interval
 * [est_c - e_c, est_c + e_c] reaches below the smallest upper bound can be the
 * argmin, and when there is more than one they are rescored exactly with
 * orc_score (the reference's own arithmetic) and compared as nearest_clusters
 * does.  The result therefore equals orc_nearest_clusters bit for bit.
 *
 * Bound (u = 2^-24, D = d): any fp32 sum of D rounded products is within
 * gamma_D sum|x_i c_i| <= gamma_D |x| |c| of the exact dot product, for the
 * reference's sequential order and for the GEMM's alike, so the two differ by
 * at most 2 gamma_D |x| |c| (gamma_D = D u / (1 - D u)).  COSINE (normalized):
 * fl(1 - s) adds u |1 - s|.  L2: |x|^2 + |c|^2 - 2 s differs from the exact sum
 * of squares by 2 gamma_D |x||c| (plus the fp64 terms), and the reference's own
 * sum of rounded squared differences is within gamma_{D+3} of it.
 * xn / cn are the fp64 norms |x|, |c|.  Metric COSINE without normalisation is
 * not covered (returns -1); call orc_nearest_clusters for it. */
int orc_assign_prefiltered(const float* S, const float* X, int64_t n, const float* C, int nlist,
                           int d, int metric, int normalized, const double* xn, const double* cn,
                           int32_t* out, int64_t* n_rescored) {
    if (metric == ORC_COSINE && !normalized) return -1;
    const double u = 1.0 / 16777216.0;
    const double g = 1.01 * (double)d * u / (1.0 - (double)d * u);
    const double g3 = 1.01 * (double)(d + 3) * u / (1.0 - (double)(d + 3) * u);
    int64_t rescored = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : rescored)
    for (int64_t i = 0; i < n; ++i) {
        const float* s = S + (size_t)i * nlist;
        const double xi = xn[i];
        /* pass 1: the smallest upper bound */
        double ub = INFINITY;
        for (int c = 0; c < nlist; ++c) {
            double est, e;
            orc_interval(metric, s[c], xi, cn[c], g, g3, &est, &e);
            if (est + e < ub) ub = est + e;
        }
        /* pass 2: candidates in ascending id order; the first one found is kept
         * unless an exact rescoring is needed */
        int32_t first = -1;
        int many = 0;
        for (int c = 0; c < nlist && !many; ++c) {
            double est, e;
            orc_interval(metric, s[c], xi, cn[c], g, g3, &est, &e);
            if (est - e <= ub) {
                if (first < 0) first = c;
                else many = 1;
            }
        }
        if (!many) {
            out[i] = first;
            continue;
        }
        /* exact rescoring of every candidate, nearest_clusters' strict '<' */
        ++rescored;
        float best = INFINITY;
        int32_t bid = -1;
        for (int c = 0; c < nlist; ++c) {
            double est, e;
            orc_interval(metric, s[c], xi, cn[c], g, g3, &est, &e);
            if (est - e > ub) continue;
            const float sc = orc_score(X + (size_t)i * d, C + (size_t)c * d, d, metric, normalized);
            if (sc < best) {
                best = sc;
                bid = c;
            }
        }
        out[i] = bid;
    }
    if (n_rescored) *n_rescored = rescored;
    return 0;
}

/* Exact unified scores of n (row, centroid) pairs: out[j] = orc_score(X[rows[j]],
 * C[cols[j]]).  Threaded over the pairs. */
void orc_score_pairs(const float* X, const int64_t* rows, const float* C, const int32_t* cols,
                     int64_t n, int d, int metric, int normalized, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; ++j)
        out[j] = orc_score(X + (size_t)rows[j] * d, C + (size_t)cols[j] * d, d, metric, normalized);
}

/* Two-means split of one list's live rows (rows in list order): the init rows are
 * orc_sample_rows(seed, n, 2); then niter E/M steps as above; out_assign gets the
 * final side (0 or 1) of each row.  Returns -1 when n < 2. */
int orc_split_2means(const float* X, int64_t n, int d, int metric, int normalized, int niter,
                     uint64_t seed, float* C2, int32_t* out_assign) {
    if (n < 2) return -1;
    return orc_kmeans_train(X, n, d, metric, normalized, 2, niter, seed, C2, out_assign);
}
