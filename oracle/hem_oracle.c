/*
 * hem_oracle.c -- CPU restatement of the reference's multilevel heavy-edge
 * matching labels (torch_fast_spdmm/torch_fast_spdmm/clustering.py:128-351,
 * cluster='hem') and of its cap enforcement (clustering.py:83-121).
 *
 * TEST INFRASTRUCTURE ONLY: the checker of the GPU labeller
 * (spmm_hem_labels); pinned against labels the reference's own clustering
 * module produced (tests/golden/clustering_golden.npz).  Written as plain
 * sequential C -- dense marker arrays, per-row candidate lists and explicit
 * scans -- for the small graphs the tests use.
 *
 * What it computes, level by level, on the binary pattern P of the current
 * (contracted) vertices:
 *   - similarity (clustering.py:128-185): columns whose degree in P exceeds
 *     hub_degree are ignored; w(i, j) = number of kept columns rows i != j
 *     share; each row keeps its topk candidates by (w desc, j asc) (topk < 0:
 *     all); the kept directed edges are united over both directions (w is
 *     symmetric, so the reference's max(G, G^T) is the union);
 *   - matching (clustering.py:188-268), up to residual_rounds rounds: every
 *     vertex picks its best live edge by (w desc, pair hash desc, j asc) --
 *     live = both ends active and, with feasible_first, the merge within the
 *     caps -- and mutual picks whose merge respects the caps are merged;
 *   - contraction (clustering.py:271-351): the smaller member of a pair stays,
 *     vertices are renumbered in index order, P's rows are united.
 *   The loop stops when a level matches nothing, one vertex is left, or after
 *   8 * max(1, ceil(log2(target))) + 16 levels.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* splitmix64-style symmetric hash of the unordered pair {a, b}, 63 bits
 * (the reference's _pair_hash, clustering.py:188-200; the constants define the
 * tie-break order, so they are the reference's). */
static int64_t pair_hash(int64_t a, int64_t b) {
    uint64_t lo = (uint64_t)(a < b ? a : b), hi = (uint64_t)(a < b ? b : a);
    uint64_t h = (lo * 0x9E3779B97F4A7C15ull) ^ (hi * 0xC2B2AE3D27D4EB4Full);
    h ^= h >> 30;
    h *= 0xBF58476D1CE4E5B9ull;
    h ^= h >> 27;
    h *= 0x94D049BB133111EBull;
    h ^= h >> 31;
    return (int64_t)(h >> 1);
}

typedef struct { int64_t j, w; } cand;

/* w descending, then j ascending */
static int cmp_cand(const void *x, const void *y) {
    const cand *a = (const cand *)x, *b = (const cand *)y;
    if (a->w != b->w) return a->w > b->w ? -1 : 1;
    return (a->j > b->j) - (a->j < b->j);
}

typedef struct { int64_t i, j, w; } edge;

static int cmp_edge(const void *x, const void *y) {
    const edge *a = (const edge *)x, *b = (const edge *)y;
    if (a->i != b->i) return a->i < b->i ? -1 : 1;
    return (a->j > b->j) - (a->j < b->j);
}

/* Similarity graph of the n-vertex pattern (ptr, idx) over m columns as CSR
 * (gptr[n + 1], gj / gw, rows ascending by j).  Returns 0, or -1 when out of
 * memory. */
static int similarity(int64_t n, int64_t m, const int64_t *ptr, const int64_t *idx, int64_t hub_degree,
                      int64_t topk, int64_t **gptr_out, int64_t **gj_out, int64_t **gw_out) {
    int64_t *deg = calloc((size_t)(m ? m : 1), sizeof(int64_t));
    int64_t *cptr = calloc((size_t)m + 1, sizeof(int64_t));
    int64_t *count = calloc((size_t)(n ? n : 1), sizeof(int64_t));
    int64_t *touched = malloc(sizeof(int64_t) * (size_t)(n ? n : 1));
    cand *cl = malloc(sizeof(cand) * (size_t)(n ? n : 1));
    int64_t ecap = 16, ne = 0;
    edge *e = malloc(sizeof(edge) * (size_t)ecap);
    int64_t *crow = NULL;
    int rc = -1;
    if (!deg || !cptr || !count || !touched || !cl || !e) goto out;
    for (int64_t k = 0; k < ptr[n]; ++k) ++deg[idx[k]];
    /* rows of each kept column (column-major copy of the pruned pattern) */
    for (int64_t c = 0; c < m; ++c) cptr[c + 1] = cptr[c] + (deg[c] <= hub_degree ? deg[c] : 0);
    crow = malloc(sizeof(int64_t) * (size_t)(cptr[m] ? cptr[m] : 1));
    if (!crow) goto out;
    {
        int64_t *fill = calloc((size_t)(m ? m : 1), sizeof(int64_t));
        if (!fill) goto out;
        for (int64_t i = 0; i < n; ++i)
            for (int64_t k = ptr[i]; k < ptr[i + 1]; ++k) {
                const int64_t c = idx[k];
                if (deg[c] <= hub_degree) crow[cptr[c] + fill[c]++] = i;
            }
        free(fill);
    }
    for (int64_t i = 0; i < n; ++i) {
        int64_t nt = 0;
        for (int64_t k = ptr[i]; k < ptr[i + 1]; ++k) {
            const int64_t c = idx[k];
            if (deg[c] > hub_degree) continue;
            for (int64_t q = cptr[c]; q < cptr[c + 1]; ++q) {
                const int64_t j = crow[q];
                if (j == i) continue;
                if (count[j]++ == 0) touched[nt++] = j;
            }
        }
        for (int64_t t = 0; t < nt; ++t) {
            cl[t].j = touched[t];
            cl[t].w = count[touched[t]];
            count[touched[t]] = 0;
        }
        qsort(cl, (size_t)nt, sizeof(cand), cmp_cand);
        const int64_t keep = topk >= 0 && topk < nt ? topk : nt;
        if (ne + 2 * keep > ecap) {
            while (ne + 2 * keep > ecap) ecap *= 2;
            edge *g = realloc(e, sizeof(edge) * (size_t)ecap);
            if (!g) goto out;
            e = g;
        }
        for (int64_t t = 0; t < keep; ++t) {
            e[ne].i = i; e[ne].j = cl[t].j; e[ne].w = cl[t].w; ++ne;
            e[ne].i = cl[t].j; e[ne].j = i; e[ne].w = cl[t].w; ++ne;
        }
    }
    qsort(e, (size_t)ne, sizeof(edge), cmp_edge);
    {
        int64_t *gptr = calloc((size_t)n + 1, sizeof(int64_t));
        int64_t *gj = malloc(sizeof(int64_t) * (size_t)(ne ? ne : 1));
        int64_t *gw = malloc(sizeof(int64_t) * (size_t)(ne ? ne : 1));
        if (!gptr || !gj || !gw) {
            free(gptr); free(gj); free(gw);
            goto out;
        }
        int64_t u = 0;
        for (int64_t k = 0; k < ne; ++k) {
            if (u > 0 && e[k].i == e[u - 1].i && e[k].j == e[u - 1].j) {
                if (e[k].w > e[u - 1].w) e[u - 1].w = e[k].w;
                continue;
            }
            e[u++] = e[k];
        }
        for (int64_t k = 0; k < u; ++k) {
            ++gptr[e[k].i + 1];
            gj[k] = e[k].j;
            gw[k] = e[k].w;
        }
        for (int64_t i = 0; i < n; ++i) gptr[i + 1] += gptr[i];
        *gptr_out = gptr;
        *gj_out = gj;
        *gw_out = gw;
    }
    rc = 0;
out:
    free(deg); free(cptr); free(count); free(touched); free(cl); free(e); free(crow);
    return rc;
}

static int within_caps(int64_t s, int64_t z, int64_t max_size, int64_t max_nnz) {
    return (max_size < 0 || s <= max_size) && (max_nnz < 0 || z <= max_nnz);
}

/* Number of label arrays a hierarchy record can hold: identity plus one per
 * level that can run. */
int64_t oracle_hem_level_slots(int64_t target) {
    int64_t lg = 0;
    while (((int64_t)1 << lg) < target) ++lg;
    return 8 * (lg > 1 ? lg : 1) + 16 + 1;
}

/*
 * labels[n]: HEM label of each row of the canonical binary pattern (indptr,
 * indices) with n rows and m columns, before cap enforcement.  max_size /
 * max_nnz / topk < 0: no cap / all candidates.  hierarchy (nullable,
 * oracle_hem_level_slots(target) x n): identity, then the labels after each
 * level that matched; *n_levels receives the number of arrays written.
 * Returns 0, or -1 when out of memory.
 */
int oracle_hem_labels(int64_t n, int64_t m, const int64_t *indptr, const int64_t *indices, int64_t target,
                      int64_t max_size, int64_t max_nnz, int64_t hub_degree, int64_t topk,
                      int32_t residual_rounds, int32_t feasible_first, int64_t *labels, int64_t *hierarchy,
                      int64_t *n_levels) {
    for (int64_t v = 0; v < n; ++v) labels[v] = v;
    int64_t rec = 0;
    if (hierarchy) memcpy(hierarchy + (rec++) * n, labels, sizeof(int64_t) * (size_t)n);
    if (n_levels) *n_levels = rec;
    if (n <= 1 || target <= 1) return 0;

    int64_t cur = n;
    int64_t *ptr = malloc(sizeof(int64_t) * (size_t)(n + 1));
    int64_t *idx = malloc(sizeof(int64_t) * (size_t)(indptr[n] ? indptr[n] : 1));
    int64_t *size = malloc(sizeof(int64_t) * (size_t)n), *nnz = malloc(sizeof(int64_t) * (size_t)n);
    int64_t *best = malloc(sizeof(int64_t) * (size_t)n), *mate = malloc(sizeof(int64_t) * (size_t)n);
    int64_t *newid = malloc(sizeof(int64_t) * (size_t)n), *mark = malloc(sizeof(int64_t) * (size_t)(m ? m : 1));
    char *active = malloc((size_t)n);
    int rc = -1;
    if (!ptr || !idx || !size || !nnz || !best || !mate || !newid || !mark || !active) goto out;
    memcpy(ptr, indptr, sizeof(int64_t) * (size_t)(n + 1));
    memcpy(idx, indices, sizeof(int64_t) * (size_t)(indptr[n] ? indptr[n] : 0));
    for (int64_t v = 0; v < n; ++v) {
        size[v] = 1;
        nnz[v] = indptr[v + 1] - indptr[v];
    }
    const int64_t levels = oracle_hem_level_slots(target) - 1;
    for (int64_t level = 0; level < levels && cur > 1; ++level) {
        int64_t *gptr = NULL, *gj = NULL, *gw = NULL;
        if (similarity(cur, m, ptr, idx, hub_degree, topk, &gptr, &gj, &gw)) goto out;
        if (gptr[cur] == 0) {
            free(gptr); free(gj); free(gw);
            break;
        }
        memset(active, 1, (size_t)cur);
        for (int64_t v = 0; v < cur; ++v) mate[v] = -1;
        int64_t matched = 0;
        for (int32_t round = 0; round < residual_rounds; ++round) {
            for (int64_t v = 0; v < cur; ++v) {
                best[v] = -1;
                if (!active[v]) continue;
                int64_t bw = 0, bh = 0;
                for (int64_t k = gptr[v]; k < gptr[v + 1]; ++k) {
                    const int64_t j = gj[k];
                    if (!active[j]) continue;
                    if (feasible_first && !within_caps(size[v] + size[j], nnz[v] + nnz[j], max_size, max_nnz))
                        continue;
                    const int64_t h = pair_hash(v, j);
                    /* candidates come in ascending j: a later one wins only when strictly better */
                    if (best[v] < 0 || gw[k] > bw || (gw[k] == bw && h > bh)) {
                        best[v] = j;
                        bw = gw[k];
                        bh = h;
                    }
                }
            }
            int64_t got = 0;
            for (int64_t v = 0; v < cur; ++v) {
                const int64_t u = best[v];
                if (u > v && best[u] == v && within_caps(size[v] + size[u], nnz[v] + nnz[u], max_size, max_nnz)) {
                    mate[v] = u;
                    mate[u] = v;
                    ++got;
                }
            }
            for (int64_t v = 0; v < cur; ++v)
                if (mate[v] >= 0) active[v] = 0;
            if (!got) break;
            matched += got;
        }
        free(gptr); free(gj); free(gw);
        if (!matched) break;
        /* contraction: the smaller member of each pair stays */
        int64_t nn = 0;
        for (int64_t v = 0; v < cur; ++v)
            if (mate[v] < 0 || mate[v] > v) newid[v] = nn++;
        for (int64_t v = 0; v < cur; ++v)
            if (mate[v] >= 0 && mate[v] < v) newid[v] = newid[mate[v]];
        int64_t *nptr = calloc((size_t)nn + 1, sizeof(int64_t));
        int64_t *nidx = malloc(sizeof(int64_t) * (size_t)(ptr[cur] ? ptr[cur] : 1));
        int64_t *nsize = calloc((size_t)nn, sizeof(int64_t)), *nz2 = calloc((size_t)nn, sizeof(int64_t));
        if (!nptr || !nidx || !nsize || !nz2) {
            free(nptr); free(nidx); free(nsize); free(nz2);
            goto out;
        }
        for (int64_t c = 0; c < m; ++c) mark[c] = -1;
        int64_t w = 0;
        for (int64_t v = 0; v < cur; ++v) {
            if (mate[v] >= 0 && mate[v] < v) continue;
            const int64_t t = newid[v];
            const int64_t mem[2] = {v, mate[v]};
            /* union of the members' sorted column lists, by a merge */
            int64_t a = ptr[v], ae = ptr[v + 1], b = 0, be = 0;
            if (mem[1] >= 0) { b = ptr[mem[1]]; be = ptr[mem[1] + 1]; }
            while (a < ae || b < be) {
                int64_t c;
                if (b >= be || (a < ae && idx[a] < idx[b])) c = idx[a++];
                else if (a >= ae || idx[b] < idx[a]) c = idx[b++];
                else { c = idx[a++]; ++b; }
                if (mark[c] != t) {
                    mark[c] = t;
                    nidx[w++] = c;
                }
            }
            nptr[t + 1] = w;
            nsize[t] = size[v] + (mem[1] >= 0 ? size[mem[1]] : 0);
            nz2[t] = nnz[v] + (mem[1] >= 0 ? nnz[mem[1]] : 0);
        }
        for (int64_t v = 0; v < n; ++v) labels[v] = newid[labels[v]];
        if (hierarchy) memcpy(hierarchy + (rec++) * n, labels, sizeof(int64_t) * (size_t)n);
        memcpy(ptr, nptr, sizeof(int64_t) * (size_t)(nn + 1));
        memcpy(idx, nidx, sizeof(int64_t) * (size_t)(w ? w : 0));
        memcpy(size, nsize, sizeof(int64_t) * (size_t)nn);
        memcpy(nnz, nz2, sizeof(int64_t) * (size_t)nn);
        free(nptr); free(nidx); free(nsize); free(nz2);
        cur = nn;
    }
    if (n_levels) *n_levels = rec;
    rc = 0;
out:
    free(ptr); free(idx); free(size); free(nnz); free(best); free(mate); free(newid); free(mark); free(active);
    return rc;
}

/*
 * Cap enforcement (clustering.py:83-121): groups are renumbered in ascending
 * label order; inside a group, members in ascending vertex order start a new
 * piece whenever adding one more would pass max_size members or max_nnz row
 * nonzeros (a piece always takes at least one member).  labels[n] are
 * rewritten with consecutive piece ids.  Caps < 0 mean none; with both absent
 * the labels are only renumbered consecutively.  Returns 0 or -1.
 */
int oracle_enforce_caps(int64_t n, int64_t *labels, const int64_t *row_nnz, int64_t max_size, int64_t max_nnz) {
    if (n <= 0) return 0;
    int64_t lmax = 0;
    for (int64_t v = 0; v < n; ++v)
        if (labels[v] > lmax) lmax = labels[v];
    int64_t *start = calloc((size_t)lmax + 2, sizeof(int64_t));
    int64_t *order = malloc(sizeof(int64_t) * (size_t)n);
    int64_t *out = malloc(sizeof(int64_t) * (size_t)n);
    if (!start || !order || !out) {
        free(start); free(order); free(out);
        return -1;
    }
    for (int64_t v = 0; v < n; ++v) ++start[labels[v] + 1];
    for (int64_t g = 0; g <= lmax; ++g) start[g + 1] += start[g];
    for (int64_t v = 0; v < n; ++v) order[start[labels[v]]++] = v;   /* ascending v per group */
    int64_t piece = -1, prev = -1, cnt = 0, load = 0;
    for (int64_t k = 0; k < n; ++k) {
        const int64_t v = order[k];
        if (labels[v] != prev) {
            prev = labels[v];
            ++piece;
            cnt = load = 0;
        } else if ((max_size >= 0 && cnt + 1 > max_size) || (max_nnz >= 0 && load + row_nnz[v] > max_nnz)) {
            ++piece;
            cnt = load = 0;
        }
        out[v] = piece;
        ++cnt;
        load += row_nnz[v];
    }
    memcpy(labels, out, sizeof(int64_t) * (size_t)n);
    free(start); free(order); free(out);
    return 0;
}
