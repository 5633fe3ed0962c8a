// spmm_boo_tc.cu -- Y = A*X for a float32 BOO matrix on the 5th-generation
// tensor cores (tcgen05, kind::tf32, three-term split for fp32 accuracy).
//
// The reference multiplies each BOO block on CUDA cores, one thread per
// (block row, feature) with the block's X rows staged in shared memory
// (torch_fast_spdmm/kernels/boo_kernel.cu:410-595).  Here a block with enough
// nonzeros is a small dense product instead: for a 128-feature tile,
//
//     Yt[f][r] += sum_c  Xt[f][c] * Ablk[r][c]        (Yt = Y^T, Xt = X^T)
//
// is a tcgen05.mma with M = 128 features, K = the block's columns in steps of
// 8.  Xt (the block's X panel, 128 features x PW columns) is the A operand in
// tensor memory; the densified block is the B operand in 128-byte-swizzled
// K-major shared memory; the accumulator Yt stays in tensor memory for the
// whole row group.  fp32 accuracy: x = hi + lo with hi = x truncated to tf32,
// Y = Xhi*Ahi + Xlo*Ahi + Xhi*Alo (the dropped lo*lo term is below
// 2^-20 |a||x|), issued as two MMAs per K step: Xhi * [Ahi; Alo] with N = 2 NR
// and Xlo * Ahi with N = NR (an M = 128 MMA costs about 50 cycles up to N ~ 96,
// so stacking saves a third of the instructions).
//
// Work decomposition: a CTA per SM runs NW independent row-group workers
// (warpgroups of 128 threads, one per quadruple of tensor-memory lane
// quadrants).  A worker owns 2 NR accumulator columns and 2 PW panel columns
// of tensor memory and two A tiles in shared memory, and processes its row
// groups end to end:
//   * the row group's blocks with >= kDenseNnz nonzeros, one after another:
//     panel loads (16-byte loads from the gathered copy below) and the scatter
//     of the block's nonzeros into an A tile overlap the MMAs of the previous
//     block; one elected thread issues the MMAs and commits to the worker's
//     mbarrier;
//   * meanwhile-free CUDA cores sum the rest -- blocks with fewer nonzeros
//     (an M = 128 MMA per 8 used columns does not pay for them) and the CSR
//     remainder (the reference's remainder kernel, boo_kernel.cu:905-937) --
//     into a shared-memory accumulator, then the COO tail (pbr_kernel.cu:
//     976-1049) and the rare products left out for non-finite operands;
//   * the accumulator comes out of tensor memory, the two sums meet, and
//     every Y element is stored once.
// Workers are independent, so four row groups proceed at once per SM and the
// tensor pipe interleaves their MMAs; there are no cross-warp queues.  Tasks
// (batch, chunk of consecutive row groups, feature tile -- innermost) are dealt
// round-robin to all workers, so they sweep the matrix together and the X
// rows they share stay in L2.
//
// Before the product a gather pass copies X column group by column group into
// Xt[batch][group][4-column quad][feature] (float4 of 4 columns), so that a
// panel row is PW/4 coalesced 16-byte loads instead of PW scattered 4-byte
// ones.
//
// Every wait is bounded (clock-limited); on expiry the worker raises an abort
// flag and stops, outstanding MMAs are drained, tensor memory is released and
// a status word readable through spmm_tc_status() is set.
#include <climits>
#include <type_traits>

#include "plan.cuh"
#include "ptx.cuh"
#include "spmm_common.cuh"

namespace spmm {

// Status word of launches given none by the caller (spmm_launch_cfg::status):
// 0, or SPMM_ETIMEOUT once a bounded wait of such a launch expired.
__device__ int g_tc_status;

namespace {

constexpr int kFeat = 128;           // features per task: MMA M, tensor-memory lanes
// Blocks with at least kDenseNnz (plan.cuh: 48) nonzeros go through the
// tensor cores; the others (and the CSR remainder) are summed on CUDA cores,
// except the ones a plan packs by quad into extra tensor-core tiles.  An M =
// 128 MMA costs ~50 cycles whatever N is, so a 32 x 32 block needs a few
// dozen nonzeros before two MMAs per 8 used columns beat per-nonzero FMAs.
constexpr int kSegs = 32;            // blocks or rows listed per pass
constexpr int kWin = 3;              // windows of 32 candidate segments loaded at once
constexpr int kListCap = 512;        // staged (row, column, value) entries per pass
constexpr int kNzPre = 4;            // nonzeros per thread fetched ahead
constexpr long long kWaitCycles = 1ll << 32;  // ~2 s at 2 GHz (default bound of a wait)

struct TcParams {
    int64_t rows, cols, K, nb, n_rg, rem_nnz, tail_nnz;
    int64_t rg_first;    // row groups [rg_first, n_rg) are multiplied (n_rg: end of the range)
    int64_t n_rg_all;    // row groups of the matrix
    const unsigned long long *cg_range;   // null, or [min, max] column group the range's blocks use
    const int32_t *rg_blk;   // plan: first block of every row group (null: search blk_row_grp)
    const uint8_t *packed;   // plan (packing): 1 for sparse blocks multiplied in packed tiles
    const int32_t *rg_slot, *slots;   // plan (packing): each group's packed quad slots
    int32_t dense_nnz;   // blocks with at least this many nonzeros use the tensor cores
    int64_t n_chunks, n_ft, n_tasks;
    int32_t chunk_rgs;
    const int32_t *row_grp_ptr, *row_ids, *col_grp_ptr, *col_ids;
    const int32_t *blk_row_grp, *blk_col_grp, *blk_nz_ptr;
    const uint8_t *blk_shift;
    const uint16_t *nz_idx;
    const float *nz_val;
    const int32_t *rem_indptr, *rem_col;
    const float *rem_val;
    const int32_t *tail_row, *tail_col;
    const float *tail_val;
    const float *X;
    float *Y;
    const float4 *Xt;  // X gathered by column group: [batch][n_cg][PW/4][K] float4
    const int32_t *x_direct;   // plan flag (or null): 1 = column order is the identity, and
                               // 64-column panels are read straight from X (no gathered copy)
    int64_t n_cg;
    int *status;          // this launch's status word (the caller's, or g_tc_status)
    long long wait_cycles;  // bound of the abortable waits, in SM clock cycles
    int32_t expire_probe;   // tests: each worker's first wait is on a barrier nothing completes
};

// One worker's shared memory.
template <int NR, int PW>
struct alignas(1024) WorkerSmem {
    static constexpr int kTileBytes = 2 * NR * PW * 4;   // [K atom][NR hi rows, NR lo rows]
    uint8_t tile[2][kTileBytes];    // A tiles (1024-aligned: 128-byte swizzle atoms)
    float ys[NR][kFeat];            // CUDA-core sums; thread f owns column f
    int2 lent[kListCap];            // staged entries: (column, value bits)
    uint8_t lrow[kListCap];
    int32_t soff[kSegs + 1];        // segment table: prefix of entry counts,
    int32_t sbase[kSegs];           //   first entry,
    int32_t scb[kSegs];             //   block: col_ids base of its group; row segment: -1
    uint32_t saux[kSegs];           //   block: index shift; row segment: local row
    int32_t scnt[kSegs];            //   entry count (while the table is filled)
    int32_t snext;                  // first segment not yet listed
    int32_t dk0[kSegs], dk1[kSegs], dcg[kSegs];  // the row group's tensor-core blocks
    uint32_t dshift[kSegs];
    uint64_t mma_bar;               // completes once per MMA commit
    uint64_t never_bar;             // never arrived on: the timeout test's wait target
    uint32_t kmask[2], aspecial[2];
};

struct Ctl {
    uint32_t tmem_base;
    volatile int abort;
};

template <int NR, int PW, int NW>
struct TcShape {
    using W = WorkerSmem<NR, PW>;
    static constexpr int kThreads = 128 * NW;
    static constexpr int kWorkerCols = 2 * NR + 2 * PW;   // accumulator + panel (hi, lo)
    static constexpr int kSmem = 1024 + NW * (int)sizeof(W) + 128;
    static constexpr uint32_t kTmemCols = 512;
    static_assert(NW * kWorkerCols <= (int)kTmemCols, "tensor memory budget");
    static_assert(NR % 16 == 0 && 2 * NR <= 256, "MMA N for M = 128");
    static_assert(PW % 32 == 0 && PW <= 64, "panel width");
    static_assert(W::kTileBytes % 1024 == 0 && sizeof(W) % 1024 == 0, "tile alignment");
    static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
    static_assert(NW <= 4, "one worker per lane-quadrant set, named barriers 1..NW");
};

// ---- bounded waits ------------------------------------------------------

__device__ __forceinline__ void raise_abort(volatile int *abort, int *status) {
    *abort = 1;
    atomicCAS(status, 0, (int)SPMM_ETIMEOUT);
}

// One poll of `bar`; the thread may sleep in the hardware until the phase
// completes or about `hint_ns` pass (no issue slots are spent meanwhile).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with the given parity; false on abort/expiry.
// Called by one thread per role (the rest of a warpgroup waits in a named
// barrier), so polling costs few issue slots.
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity, volatile int *abort, int *status,
                                           long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 16; ++i)
            if (mbar_try_wait_sleep(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > limit) {
            raise_abort(abort, status);
            return false;
        }
    }
}

// OR of `v` over the `n` threads of named barrier `id` (also a barrier).
__device__ __forceinline__ bool bar_or(uint32_t id, uint32_t n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "barrier.cta.red.or.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

// AND of `v` over the `n` threads of named barrier `id` (also a barrier).
__device__ __forceinline__ bool bar_and(uint32_t id, uint32_t n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "barrier.cta.red.and.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

// ---- operand layout -------------------------------------------------------

// Byte offset of Ahi(r, c) in a block tile stored K-major with the 128-byte
// swizzle: 32 columns (128 B) per row and atom of 8 rows, the 16-byte chunk
// index XORed with the row within the atom.  Each 32-column K atom holds the
// NR hi rows followed by the NR lo rows (Alo(r, c) = Ahi offset + NR * 128),
// so one descriptor spans the stacked [Ahi; Alo] operand of an N = 2 NR MMA.
template <int NR>
__device__ __forceinline__ uint32_t a_offset(uint32_t r, uint32_t c) {
    const uint32_t cc = c & 31u;
    return (c >> 5) * (2u * NR * 128u) + r * 128u + ((((cc >> 2) ^ r) & 7u) << 4) + ((cc & 3u) << 2);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 B apart (stride byte offset), leading byte offset unused (16 B).
__device__ __forceinline__ uint64_t b_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::tf32: fp32 accumulate, A = B = tf32, both
// K-major, M = 128, N = NR.
template <int NR>
__host__ __device__ constexpr uint32_t idesc_tf32() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(NR >> 3) << 17) | ((uint32_t)(kFeat >> 4) << 24);
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

__device__ __forceinline__ bool finite(float x) { return fabsf(x) <= 3.402823466e38f; }


// ---- the worker ----------------------------------------------------------------

// Waits for the phase of `bar` with the given parity, bounded by the clock
// only (used to drain MMAs before tensor memory is released, also after an
// abort).
__device__ __forceinline__ bool drain_phase(uint64_t *bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}

// CUDA-core part of a row group, summed into w.ys (thread f owns column f):
// the entries of its blocks with fewer than dense_nnz nonzeros, then its
// rows' CSR remainder.  Segments (one per block or row) are listed by warp 0
// (seg_table), their entries staged as (local row, column, value) by the
// warpgroup (stage), and each thread sums them for its feature (sum_range).

// Segment table (warp 0): the next kSegs NON-EMPTY segments from segment
// `pos` on, in segment order, and in w.snext the segment to resume from.
// Candidates are loaded kWin x 32 at a time in two rounds of independent
// loads (more windows spill registers at four workers per SM), so rows
// without remainder entries and tensor-core blocks cost no pass of their own
// and a row group's segment list costs one load chain, not one per 32
// (64-row groups with a remainder: three passes became one).
template <int NR, int PW>
__device__ __forceinline__ void seg_table(const TcParams &p, WorkerSmem<NR, PW> &w, int64_t bs, int nblk, int nseg,
                                          int32_t rbase, int pos, int wt) {
    if (wt >= 32) return;
    const unsigned lt = lanemask_lt();
    int filled = 0;
    while (filled < kSegs && pos < nseg) {
        // candidate s = pos + 32 u + lane: block s (s < nblk; empty when it goes
        // through the tensor cores) or the CSR remainder of local row s - nblk.
        // Two rounds of independent loads for all windows.
        int32_t t0[kWin], t1[kWin], t2[kWin];
#pragma unroll
        for (int u = 0; u < kWin; ++u) {
            const int sc = pos + 32 * u + wt;
            t0[u] = t1[u] = t2[u] = 0;
            if (sc < nblk) {
                const int64_t b = bs + sc;
                t0[u] = __ldg(p.blk_nz_ptr + b);
                t1[u] = __ldg(p.blk_nz_ptr + b + 1);
                t2[u] = __ldg(p.blk_col_grp + b);
            } else if (sc < nseg) {
                t2[u] = __ldg(p.row_ids + rbase + (sc - nblk));
            }
        }
        int cnt[kWin], base[kWin], cb[kWin];
        uint32_t aux[kWin];
#pragma unroll
        for (int u = 0; u < kWin; ++u) {
            const int sc = pos + 32 * u + wt;
            cnt[u] = 0;
            base[u] = 0;
            cb[u] = -1;
            aux[u] = 0;
            if (sc < nblk) {
                if (t1[u] - t0[u] < p.dense_nnz && !(p.packed && __ldg(p.packed + bs + sc))) {
                    cnt[u] = t1[u] - t0[u];
                    base[u] = t0[u];
                    cb[u] = __ldg(p.col_grp_ptr + t2[u]);
                    aux[u] = __ldg(p.blk_shift + bs + sc);
                }
            } else if (sc < nseg) {
                base[u] = __ldg(p.rem_indptr + t2[u]);
                cnt[u] = __ldg(p.rem_indptr + t2[u] + 1) - base[u];
                aux[u] = (uint32_t)(sc - nblk);
            }
        }
        int next = pos;   // first candidate not consumed
#pragma unroll
        for (int u = 0; u < kWin; ++u) {
            if (filled < kSegs) {
                const unsigned ne = __ballot_sync(kFullMask, cnt[u] > 0);
                const int room = kSegs - filled;
                const int rank = __popc(ne & lt);
                if (cnt[u] > 0 && rank < room) {
                    const int slot = filled + rank;
                    w.scnt[slot] = cnt[u];
                    w.sbase[slot] = base[u];
                    w.scb[slot] = cb[u];
                    w.saux[slot] = aux[u];
                }
                if (__popc(ne) > room) {   // full: resume at the first candidate not taken
                    const unsigned first_left = __ballot_sync(kFullMask, cnt[u] > 0 && rank == room);
                    next = pos + 32 * u + (__ffs(first_left) - 1);
                    filled = kSegs;
                } else {                   // the whole window of 32 is consumed
                    filled += __popc(ne);
                    next = pos + 32 * (u + 1);
                }
            }
        }
        pos = next;
    }
    __syncwarp();
    int incl = wt < filled ? w.scnt[wt] : 0;
    if (wt >= filled) {   // unused slots: empty segments
        w.sbase[wt] = 0;
        w.scb[wt] = -1;
        w.saux[wt] = 0;
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(kFullMask, incl, o);
        if (wt >= o) incl += n;
    }
    w.soff[wt + 1] = incl;
    if (wt == 0) {
        w.soff[0] = 0;
        w.snext = pos < nseg ? pos : nseg;
    }
}


// Entries [g0, g0 + ne) of the current segment table into the list.
template <int NR, int PW>
__device__ __forceinline__ void stage(const TcParams &p, WorkerSmem<NR, PW> &w, int g0, int ne, int wt) {
    for (int i = wt; i < ne; i += 128) {
        const int g = g0 + i;
        int lo = 0, hi = kSegs - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (w.soff[mid] <= g) lo = mid; else hi = mid - 1;
        }
        const int kidx = w.sbase[lo] + (g - w.soff[lo]);
        uint32_t r;
        int32_t col;
        float v;
        if (w.scb[lo] >= 0) {
            const uint32_t idx = __ldg(p.nz_idx + kidx), sh = w.saux[lo];
            r = idx >> sh;
            col = __ldg(p.col_ids + w.scb[lo] + (int32_t)(idx & ((1u << sh) - 1u)));
            v = __ldg(p.nz_val + kidx);
        } else {
            r = w.saux[lo];
            col = __ldg(p.rem_col + kidx);
            v = __ldg(p.rem_val + kidx);
        }
        w.lrow[i] = (uint8_t)(r < (uint32_t)NR ? r : 255u);
        w.lent[i] = make_int2(col, __float_as_int(v));
    }
}

// List entries [i0, i1) into ys for this thread's feature (i0 a multiple of
// 4).  Entries of a block arrive row by row: a running sum per row run, added
// to ys when the row changes (no shared-memory dependency chain between
// consecutive entries); 16 X loads in flight, the entries held in registers
// across the ys updates and their rows read four to a word.
template <int NR, int PW>
__device__ __forceinline__ void sum_range(const TcParams &p, WorkerSmem<NR, PW> &w, int i0, int i1, const float *xb,
                                          int wt) {
    constexpr int U = 16;
    uint32_t cur = 255u;
    float run = 0.f;
    auto add = [&](uint32_t r, float v, float x) {
        if (r != cur) {
            if (cur < (uint32_t)NR) w.ys[cur][wt] += run;
            cur = r;
            run = 0.f;
        }
        run = fmaf(v, x, run);
    };
    int i = i0;
    for (; i + U <= i1; i += U) {
        float x[U];
        int2 en[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            en[u] = w.lent[i + u];
            x[u] = __ldg(xb + (int64_t)en[u].x * p.K);
        }
#pragma unroll
        for (int u = 0; u < U; u += 4) {
            const uint32_t r4 = *reinterpret_cast<const uint32_t *>(&w.lrow[i + u]);
#pragma unroll
            for (int q = 0; q < 4; ++q) add((r4 >> (8 * q)) & 0xFFu, __int_as_float(en[u + q].y), x[u + q]);
        }
    }
    for (; i < i1; ++i) {
        const int2 en = w.lent[i];
        add(w.lrow[i], __int_as_float(en.y), __ldg(xb + (int64_t)en.x * p.K));
    }
    if (cur < (uint32_t)NR) w.ys[cur][wt] += run;
}

// The whole CUDA-core part, pass by pass (row groups whose entries do not fit
// one segment table and list).
template <int NR, int PW>
__device__ __forceinline__ void cuda_part(const TcParams &p, WorkerSmem<NR, PW> &w, int64_t bs, int64_t be,
                                          int32_t rbase, int32_t nr, const float *xb, int wt, uint32_t bar) {
    const int nblk = (int)(be - bs);
    const int nseg = nblk + (p.rem_nnz ? (nr < NR ? nr : NR) : 0);
    for (int pos = 0; pos < nseg;) {
        seg_table<NR, PW>(p, w, bs, nblk, nseg, rbase, pos, wt);
        named_bar_sync(bar, 128);
        const int total = w.soff[kSegs];
        pos = w.snext;
        for (int g0 = 0; g0 < total; g0 += kListCap) {
            const int ne = total - g0 < kListCap ? total - g0 : kListCap;
            stage<NR, PW>(p, w, g0, ne, wt);
            named_bar_sync(bar, 128);
            sum_range<NR, PW>(p, w, 0, ne, xb, wt);
            named_bar_sync(bar, 128);  // the list is reused by the next pass
        }
        named_bar_sync(bar, 128);      // the segment table is rewritten next
    }
}

// Rare contributions, summed into w.ys by each thread for its feature: the
// tensor-core block products left out for a non-finite operand (`special`),
// and the COO tail (the reference's tail kernel, pbr_kernel.cu:976-1049).
// Rolled loops: the hot path stays small for the instruction cache.
template <int NR, int PW>
__device__ __forceinline__ void rare_part(const TcParams &p, WorkerSmem<NR, PW> &w, int64_t bs, int64_t be,
                                          int32_t rbase, int32_t nr, bool special, const float *xb, int wt) {
    if (special) {
        for (int64_t b = bs; b < be; ++b) {
            const int32_t k0 = __ldg(p.blk_nz_ptr + b), k1 = __ldg(p.blk_nz_ptr + b + 1);
            if (k1 - k0 < p.dense_nnz && !(p.packed && __ldg(p.packed + b))) continue;   // on CUDA cores
            const uint32_t shift = __ldg(p.blk_shift + b), cm = (1u << shift) - 1u;
            const int32_t cbase = __ldg(p.col_grp_ptr + __ldg(p.blk_col_grp + b));
            for (int32_t k = k0; k < k1; ++k) {
                const uint32_t idx = __ldg(p.nz_idx + k);
                const uint32_t r = idx >> shift;
                const float a = __ldg(p.nz_val + k);
                const float x = __ldg(xb + (int64_t)__ldg(p.col_ids + cbase + (int32_t)(idx & cm)) * p.K);
                if (r < (uint32_t)NR && (!finite(a) || !finite(x))) w.ys[r][wt] = fmaf(a, x, w.ys[r][wt]);
            }
        }
    }
    if (!p.tail_nnz) return;
    for (int32_t r = 0; r < nr && r < NR; ++r) {
        const int32_t row = __ldg(p.row_ids + rbase + r);
        int64_t lo = 0, hi = p.tail_nnz;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (__ldg(p.tail_row + mid) < row) lo = mid + 1; else hi = mid;
        }
        float a = w.ys[r][wt];
        for (int64_t k = lo; k < p.tail_nnz && __ldg(p.tail_row + k) == row; ++k)
            a = fmaf(__ldg(p.tail_val + k), __ldg(xb + (int64_t)__ldg(p.tail_col + k) * p.K), a);
        w.ys[r][wt] = a;
    }
}

// Rows NR, 2 NR, ... of a row group larger than NR (no kept blocks there):
// their CSR remainder and COO tail on CUDA cores, NR rows at a time.  Kept out
// of line: it is rare, and the worker's registers stay for the common case.
template <int NR, int PW>
__device__ __noinline__ void large_group_rows(const TcParams &p, WorkerSmem<NR, PW> &w, int64_t b, int32_t rbase,
                                              int32_t nr, const float *xb, float *yb, int wt, uint32_t bar) {
    for (int32_t r0 = NR; r0 < nr; r0 += NR) {
        const int32_t rb = rbase + r0, nrc = nr - r0 < NR ? nr - r0 : NR;
        for (int r = 0; r < NR; ++r) w.ys[r][wt] = 0.f;
        if (p.rem_nnz) cuda_part<NR, PW>(p, w, b, b, rb, nrc, xb, wt, bar);
        if (p.tail_nnz) rare_part<NR, PW>(p, w, b, b, rb, nrc, false, xb, wt);
        for (int r = 0; r < nrc; ++r) __stcs(yb + (int64_t)__ldg(p.row_ids + rb + r) * p.K, w.ys[r][wt]);
    }
}

// One row-group worker (a warpgroup; wt = thread in the worker, tensor-memory
// lane wt).  `tcol`: first of its 2 NR accumulator + 2 PW panel columns.
template <int NR, int PW, bool SPLIT>
__device__ void worker(const TcParams &p, WorkerSmem<NR, PW> &w, Ctl &ctl, uint32_t tcol, int64_t wid,
                       int64_t nworkers, int wt, uint32_t bar) {
    constexpr int KS = PW / 8;
    constexpr int RH = (NR + 31) / 32;
    constexpr uint32_t idesc1 = idesc_tf32<NR>();       // N = NR: Xlo * Ahi
    constexpr uint32_t idesc2 = idesc_tf32<2 * NR>();   // N = 2 NR: Xhi * [Ahi; Alo]
    volatile int *abort = &ctl.abort;
    const int lane = wt & 31;
    const uint32_t lane_addr = (uint32_t)((wt & ~31) << 16);
    const uint32_t dacc = tcol, xslot = tcol + 2 * NR;
    uint32_t ncommit = 0;   // commits to w.mma_bar (one per tensor-core block)
    bool ok = true;

    // Thread 0 waits, the warpgroup learns the (uniform) outcome at a barrier.
    // With expire_probe (tests of the timeout path) the first wait is on a
    // barrier that nothing arrives on, so it expires after wait_cycles.
    bool probe = p.expire_probe != 0;
    auto wait_commit = [&](uint32_t c) -> bool {
        bool r = true;
        if (wt == 0) {
            if (probe) r = wait_phase(&w.never_bar, 0u, abort, p.status, p.wait_cycles);
            if (r) r = wait_phase(&w.mma_bar, c & 1u, abort, p.status, p.wait_cycles);
        }
        probe = false;
        return bar_and(bar, 128, r);
    };
    auto prefetch = [&](int i, uint16_t (&ip)[kNzPre], float (&vp)[kNzPre]) {
        const int32_t k0 = w.dk0[i], n = w.dk1[i] - k0;
#pragma unroll
        for (int u = 0; u < kNzPre; ++u) {
            const int e = wt + 128 * u;
            ip[u] = e < n ? __ldg(p.nz_idx + k0 + e) : (uint16_t)0;
            vp[u] = e < n ? __ldg(p.nz_val + k0 + e) : 0.f;
        }
    };

    for (int64_t task = wid; task < p.n_tasks && ok; task += nworkers) {
        const int64_t ft = task % p.n_ft, chunk = (task / p.n_ft) % p.n_chunks;
        const int64_t bt = task / (p.n_ft * p.n_chunks);
        const int64_t rg0 = p.rg_first + chunk * p.chunk_rgs;
        const int64_t rg1 = rg0 + p.chunk_rgs < p.n_rg ? rg0 + p.chunk_rgs : p.n_rg;
        const float *xb = p.X + bt * p.cols * p.K + ft * kFeat + wt;
        float *yb = p.Y + bt * p.rows * p.K + ft * kFeat + wt;
        const float4 *xt = p.Xt + bt * p.n_cg * (PW / 4) * p.K + ft * kFeat + wt;
        // 64-column panels of an identity column order come straight from X
        // (64 4-byte loads per lane instead of 16 16-byte ones from the gathered
        // copy, and no gather pass: measured faster at PW = 64, C4 1.51 ->
        // 1.34 ms; at PW = 32, C2, the gathered copy stays faster)
        const bool direct = PW == 64 && p.x_direct && __ldg(p.x_direct) != 0;
        int64_t b = p.rg_blk ? (int64_t)__ldg(p.rg_blk + rg0)
                             : warp_lower_bound(p.blk_row_grp, p.nb, rg0, lane);   // every warp: same answer
        for (int64_t rg = rg0; rg < rg1 && ok; ++rg) {
            const int64_t be = p.rg_blk ? (int64_t)__ldg(p.rg_blk + rg + 1) : group_end(p.blk_row_grp, p.nb, b, rg, lane);
            const int32_t rbase = __ldg(p.row_grp_ptr + rg);
            const int32_t nr = __ldg(p.row_grp_ptr + rg + 1) - rbase;
            uint32_t started = 0;
            bool special = false, sparse = false;
            uint16_t i1[kNzPre], i2[kNzPre];
            float v1[kNzPre], v2[kNzPre];
            // One tensor-core tile: dense block i of the listing (ns == 0), or a
            // packed tile of ns quad slots, listed as (first entry, end, Xt quad
            // index, shift | quad << 8) in dk0 / dk1 / dcg / dshift.  False on abort.
            auto tile_step = [&](auto packed_tile, int i, int ns, bool has_next) -> bool {
                constexpr bool PACKED = decltype(packed_tile)::value;
                const int t = (int)(ncommit & 1u);
                uint8_t *tile = w.tile[t];
                // 1. the panel: 16-byte loads of the tile's quads
                float x[PW];
                if constexpr (!PACKED) {
                    if (direct) {   // identity column order: the group's columns are consecutive X rows
                        const int32_t g = w.dcg[i];
                        const int32_t c0 = __ldg(p.col_grp_ptr + g), nc = __ldg(p.col_grp_ptr + g + 1) - c0;
                        const float *xc = xb + (int64_t)c0 * p.K;
#pragma unroll
                        for (int c = 0; c < PW; ++c) x[c] = c < nc ? __ldg(xc + (int64_t)c * p.K) : 0.f;
                    } else {
                        const float4 *xq = xt + (int64_t)w.dcg[i] * (PW / 4) * p.K;
#pragma unroll
                        for (int q = 0; q < PW / 4; ++q) {
                            const float4 a = __ldg(xq + q * p.K);
                            x[4 * q] = a.x; x[4 * q + 1] = a.y; x[4 * q + 2] = a.z; x[4 * q + 3] = a.w;
                        }
                    }
                    // 2. next block's nonzeros
                    if (has_next) prefetch(i + 1, i2, v2);
                } else {
                    if (direct) {   // slot q: quad qd of group g, columns c0 + 4 qd + j of the group
#pragma unroll
                        for (int q = 0; q < PW / 4; ++q) {
                            const int32_t g = q < ns ? w.dcg[q] / (PW / 4) : 0, qd = q < ns ? w.dcg[q] % (PW / 4) : 0;
                            const int32_t c0 = q < ns ? __ldg(p.col_grp_ptr + g) : 0;
                            const int32_t nc = q < ns ? __ldg(p.col_grp_ptr + g + 1) - c0 : 0;
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                x[4 * q + j] = 4 * qd + j < nc ? __ldg(xb + (int64_t)(c0 + 4 * qd + j) * p.K) : 0.f;
                        }
                    } else {
#pragma unroll
                        for (int q = 0; q < PW / 4; ++q) {
                            const float4 a = q < ns ? __ldg(xt + (int64_t)w.dcg[q] * p.K) : make_float4(0.f, 0.f, 0.f, 0.f);
                            x[4 * q] = a.x; x[4 * q + 1] = a.y; x[4 * q + 2] = a.z; x[4 * q + 3] = a.w;
                        }
                    }
                }
                // 3. zero the tile (its MMAs, two tiles back, are complete) and scatter
                {
                    float4 *z = reinterpret_cast<float4 *>(tile);
#pragma unroll
                    for (int u = 0; u < WorkerSmem<NR, PW>::kTileBytes / 16 / 128; ++u)
                        z[wt + 128 * u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (wt == 0) {
                        w.kmask[t] = 0u;
                        w.aspecial[t] = 0u;
                    }
                    named_bar_sync(bar, 128);
                    uint32_t m = 0u;
                    bool asp = false;
                    auto place = [&](uint32_t r, uint32_t c, float v) {
                        if (r < (uint32_t)NR && c < (uint32_t)PW) {
                            if (!finite(v)) {
                                asp = true;
                                v = 0.f;
                            }
                            const uint32_t off = a_offset<NR>(r, c);
                            if constexpr (SPLIT) {
                                const float h = tf32_hi(v);
                                *reinterpret_cast<float *>(tile + off) = h;
                                *reinterpret_cast<float *>(tile + NR * 128 + off) = v - h;
                            } else {   // one tf32 term: the tensor cores read the value's tf32 part
                                *reinterpret_cast<float *>(tile + off) = v;
                            }
                            m |= 1u << (c >> 3);
                        }
                    };
                    if constexpr (!PACKED) {
                        const uint32_t shift = w.dshift[i], cm = (1u << shift) - 1u;
                        auto put = [&](uint32_t idx, float v) { place(idx >> shift, idx & cm, v); };
                        const int32_t k0 = w.dk0[i];
                        const int n = w.dk1[i] - k0;
#pragma unroll
                        for (int u = 0; u < kNzPre; ++u)
                            if (wt + 128 * u < n) put(i1[u], v1[u]);
                        // large blocks: the rest in batches of 8 loads in flight
                        for (int e0 = wt + 128 * kNzPre; e0 < n; e0 += 128 * 8) {
                            uint16_t ib[8];
                            float vb[8];
#pragma unroll
                            for (int u = 0; u < 8; ++u) {
                                const int e = e0 + 128 * u;
                                ib[u] = e < n ? __ldg(p.nz_idx + k0 + e) : (uint16_t)0;
                                vb[u] = e < n ? __ldg(p.nz_val + k0 + e) : 0.f;
                            }
#pragma unroll
                            for (int u = 0; u < 8; ++u)
                                if (e0 + 128 * u < n) put(ib[u], vb[u]);
                        }
                    } else {
                        // slot s's entries in its quad go to columns 4 s .. 4 s + 3
                        constexpr int TPS = 128 / (PW / 4);   // threads per slot
                        const int sl = wt / TPS, tt = wt % TPS;
                        if (sl < ns) {
                            const uint32_t sh = w.dshift[sl] & 0xFFu, qd = w.dshift[sl] >> 8, cm = (1u << sh) - 1u;
                            const int32_t e1 = w.dk1[sl];
                            for (int32_t e = w.dk0[sl] + tt; e < e1; e += TPS) {
                                const uint32_t idx = __ldg(p.nz_idx + e), c = idx & cm;
                                if ((c >> 2) == qd) place(idx >> sh, 4u * (uint32_t)sl + (c & 3u), __ldg(p.nz_val + e));
                            }
                        }
                    }
                    m = __reduce_or_sync(kFullMask, m);
                    if (lane == 0 && m) atomicOr(&w.kmask[t], m);
                    if (__any_sync(kFullMask, asp) && lane == 0) w.aspecial[t] = 1u;
                }
                // 4. the previous tile's MMAs are done: the panel slot is free
                if (ncommit > 0 && !wait_commit(ncommit - 1)) return false;
                if (ncommit == 0) named_bar_sync(bar, 128);
                tc_fence_after();
                const uint32_t kmask = w.kmask[t];
                // 5. split and store the panel: hi at xslot, lo at xslot + PW
                // x * 0 is NaN exactly for a non-finite x: one FMA per value
                // detects them; the rare panel that has one is cleaned
                float chk = 0.f;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks)
                    if (kmask & (1u << ks))
#pragma unroll
                        for (int e = 0; e < 8; ++e) chk = fmaf(x[ks * 8 + e], 0.f, chk);
                const bool xsp = chk != chk;
                if (xsp) {
#pragma unroll
                    for (int c = 0; c < PW; ++c)
                        if (!finite(x[c])) x[c] = 0.f;
                }
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    if (kmask & (1u << ks)) {
                        uint32_t h[8], l[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float v = x[ks * 8 + e];
                            const float hv = SPLIT ? tf32_hi(v) : v;
                            h[e] = __float_as_uint(hv);
                            l[e] = __float_as_uint(v - hv);
                        }
                        tmem_st8(xslot + lane_addr + ks * 8, h);
                        if constexpr (SPLIT) tmem_st8(xslot + lane_addr + PW + ks * 8, l);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                fence_proxy_async_smem();
                if (bar_or(bar, 128, xsp) || w.aspecial[t]) special = true;
                // 6. MMAs of the tile, issued by one thread
                if (wt == 0) {
                    tc_fence_after();
                    const uint64_t bd = b_desc_sw128(smem_u32(tile));
                    uint32_t accum = started;   // 0: the first MMA of the group overwrites
#pragma unroll
                    for (int ks = 0; ks < KS; ++ks) {
                        if (kmask & (1u << ks)) {
                            const uint64_t bh = bd + (uint64_t)(((ks >> 2) * (2 * NR * 128) + (ks & 3) * 32) >> 4);
                            if constexpr (SPLIT) {
                                mma_tf32_ts(dacc, xslot + ks * 8, bh, idesc2, accum);
                                mma_tf32_ts(dacc, xslot + PW + ks * 8, bh, idesc1, 1u);
                            } else {
                                mma_tf32_ts(dacc, xslot + ks * 8, bh, idesc1, accum);
                            }
                            accum = 1;
                        }
                    }
                    mma_commit(&w.mma_bar);
                }
                if (kmask) started = 1;   // uniform: every thread read kmask
                ++ncommit;
                if constexpr (!PACKED) {
#pragma unroll
                    for (int u = 0; u < kNzPre; ++u) {
                        i1[u] = i2[u];
                        v1[u] = v2[u];
                    }
                }
                return true;
            };
            // ---- dense blocks, listed kSegs blocks at a time ----
            for (int64_t b0 = b; b0 < be && ok; b0 += kSegs) {
                const int nblk = be - b0 < kSegs ? (int)(be - b0) : kSegs;
                int nd;
                {
                    const int64_t bb = b0 + lane;
                    int32_t k0 = 0, k1 = 0;
                    if (lane < nblk) {
                        k0 = __ldg(p.blk_nz_ptr + bb);
                        k1 = __ldg(p.blk_nz_ptr + bb + 1);
                    }
                    const bool dense = lane < nblk && k1 - k0 >= p.dense_nnz;
                    const bool pk = p.packed && lane < nblk && !dense && __ldg(p.packed + bb);
                    const unsigned dm = __ballot_sync(kFullMask, dense);
                    nd = __popc(dm);
                    if (nd + __popc(__ballot_sync(kFullMask, pk)) < nblk) sparse = true;   // CUDA-core blocks
                    if (wt < 32 && dense) {
                        const int slot = __popc(dm & ((1u << lane) - 1u));
                        w.dk0[slot] = k0;
                        w.dk1[slot] = k1;
                        w.dcg[slot] = __ldg(p.blk_col_grp + bb);
                        w.dshift[slot] = __ldg(p.blk_shift + bb);
                    }
                }
                named_bar_sync(bar, 128);
                if (nd > 0) prefetch(0, i1, v1);
                for (int i = 0; i < nd && ok; ++i) ok = tile_step(std::false_type{}, i, 0, i + 1 < nd);
            }
            // ---- packed tiles: quads of the group's packed sparse blocks ----
            if (p.rg_slot && ok) {
                const int32_t s0 = __ldg(p.rg_slot + rg), s1 = __ldg(p.rg_slot + rg + 1);
                for (int32_t t0 = s0; t0 < s1 && ok; t0 += PW / 4) {
                    const int ns = s1 - t0 < PW / 4 ? s1 - t0 : PW / 4;
                    if (wt < ns) {
                        const int32_t sl = __ldg(p.slots + t0 + wt);
                        const int64_t bb = sl >> 4;
                        const uint32_t qd = (uint32_t)(sl & 15);
                        w.dk0[wt] = __ldg(p.blk_nz_ptr + bb);
                        w.dk1[wt] = __ldg(p.blk_nz_ptr + bb + 1);
                        w.dcg[wt] = __ldg(p.blk_col_grp + bb) * (PW / 4) + (int32_t)qd;
                        w.dshift[wt] = (uint32_t)__ldg(p.blk_shift + bb) | (qd << 8);
                    }
                    named_bar_sync(bar, 128);
                    ok = tile_step(std::true_type{}, 0, ns, false);
                }
            }
            if (!ok) break;
            const bool any_dense = started != 0;
            const int32_t nrc = nr < NR ? nr : NR;
            int32_t myrow[RH];
#pragma unroll
            for (int h = 0; h < RH; ++h) {
                const int r = h * 32 + lane;
                myrow[h] = r < nrc ? __ldg(p.row_ids + rbase + r) : -1;
            }
            // ---- CUDA-core part (overlaps the last block's MMAs) ----
            const bool cpart = sparse || p.rem_nnz;
            bool in_ys = cpart || p.tail_nnz;
            if (in_ys) {
#pragma unroll
                for (int r = 0; r < NR; ++r) w.ys[r][wt] = 0.f;
                if (cpart) cuda_part<NR, PW>(p, w, b, be, rbase, nrc, xb, wt, bar);
            }
            // ---- the accumulator ----
            float acc[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] = 0.f;
            if (any_dense) {
                if (!(ok = wait_commit(ncommit - 1))) break;
                tc_fence_after();
#pragma unroll
                for (int h = 0; h < NR / 16; ++h) {
                    uint32_t v[16], u[16];
                    const uint32_t a0 = dacc + lane_addr + h * 16;
                    tmem_ld16(a0, v);
                    if constexpr (SPLIT) tmem_ld16(a0 + NR, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        acc[h * 16 + q] = SPLIT ? __uint_as_float(v[q]) + __uint_as_float(u[q]) : __uint_as_float(v[q]);
                }
                tc_fence_before();
            }
            if (special || p.tail_nnz) {
                if (!in_ys) {
#pragma unroll
                    for (int r = 0; r < NR; ++r) w.ys[r][wt] = 0.f;
                    in_ys = true;
                }
                rare_part<NR, PW>(p, w, b, be, rbase, nrc, special, xb, wt);
            }
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const int32_t row = __shfl_sync(kFullMask, myrow[r / 32], r % 32);
                if (row >= 0) __stcs(yb + (int64_t)row * p.K, in_ys ? w.ys[r][wt] + acc[r] : acc[r]);
            }
            // A row group with a kept block has at most max_nr <= NR rows; a
            // larger one (its blocks all spilled, or an empty group under KEEP)
            // holds only CSR remainder and COO tail entries past row NR.
            if (nr > NR) large_group_rows<NR, PW>(p, w, b, rbase, nr, xb, yb, wt, bar);
            b = be;
        }
    }
    // drain: every MMA issued by this worker completes before tensor memory is released
    if (wt == 0 && ncommit > 0) drain_phase(&w.mma_bar, (ncommit - 1) & 1u);
}

template <int NR, int PW, int NW, bool SPLIT>
__global__ void __launch_bounds__(TcShape<NR, PW, NW>::kThreads, 1) boo_tc_kernel(const __grid_constant__ TcParams p) {
    using Shape = TcShape<NR, PW, NW>;
    using W = WorkerSmem<NR, PW>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    W *ws = reinterpret_cast<W *>(base);
    Ctl &ctl = *reinterpret_cast<Ctl *>(base + NW * sizeof(W));
    const int tid = threadIdx.x, warp = tid >> 5, wk = warp >> 2;

    if (tid == 0) {
        for (int k = 0; k < NW; ++k) {
            mbar_init(&ws[k].mma_bar, 1);
            mbar_init(&ws[k].never_bar, 1);
        }
        ctl.abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&ctl.tmem_base, Shape::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl.tmem_base;

    worker<NR, PW, SPLIT>(p, ws[wk], ctl, tmem + (uint32_t)(wk * Shape::kWorkerCols), (int64_t)blockIdx.x * NW + wk,
                   (int64_t)gridDim.x * NW, tid & 127, 1u + (uint32_t)wk);

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Shape::kTmemCols);
    }
}

// Gather pass: Xt[bt][g][q][f] = (X[bt][col 4q..4q+3 of group g][f]) as one
// float4, zeros past the group's size.  One CTA per (bt, g): the group's row
// pointers in shared memory, then each thread writes float4s of two quads at
// a time (16 X loads in flight per thread at K = 128); reads and writes are
// coalesced over f.  HBM-bound streaming copy.
template <int PW>
__global__ void __launch_bounds__(256) boo_gather_kernel(const TcParams p) {
    constexpr int QW = PW / 4;
    __shared__ const float *xr[PW];
    if (PW == 64 && p.x_direct && __ldg(p.x_direct) != 0) return;   // the worker reads X itself
    const int64_t g = blockIdx.x % p.n_cg, bt = blockIdx.x / p.n_cg;
    if (threadIdx.x < PW) {
        const int32_t cbase = __ldg(p.col_grp_ptr + g);
        const int32_t nc = __ldg(p.col_grp_ptr + g + 1) - cbase;
        const int c = threadIdx.x;
        xr[c] = c < nc ? p.X + (bt * p.cols + __ldg(p.col_ids + cbase + c)) * p.K : nullptr;
    }
    __syncthreads();
    if (p.cg_range && (g < (int64_t)p.cg_range[0] || g > (int64_t)p.cg_range[1])) return;   // not used
    float4 *out = const_cast<float4 *>(p.Xt) + (bt * p.n_cg + g) * QW * p.K;
    // item = (quad q, 4 features from f): four 16-byte loads (one per column
    // of the quad), a 4 x 4 transpose in registers, four 16-byte stores
    const int64_t f4 = p.K / 4;
    for (int64_t it = threadIdx.x; it < QW * f4; it += blockDim.x) {
        const int q = (int)(it / f4);
        const int64_t f = (it % f4) * 4;
        float4 v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float *r = xr[4 * q + c];
            v[c] = r ? __ldg(reinterpret_cast<const float4 *>(r + f)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float4 *o = out + q * p.K + f;
        o[0] = make_float4(v[0].x, v[1].x, v[2].x, v[3].x);
        o[1] = make_float4(v[0].y, v[1].y, v[2].y, v[3].y);
        o[2] = make_float4(v[0].z, v[1].z, v[2].z, v[3].z);
        o[3] = make_float4(v[0].w, v[1].w, v[2].w, v[3].w);
    }
}

// Smallest and largest column group used by the blocks of row groups
// [rg_first, n_rg) into cg_range[0] / [1] (initialised to ~0 / 0 by the host),
// so that a row-group-range product gathers only those groups.
__global__ void __launch_bounds__(256) cg_range_kernel(const TcParams p, unsigned long long *cg_range) {
    const int lane = threadIdx.x & 31;
    const int64_t b0 = warp_lower_bound(p.blk_row_grp, p.nb, p.rg_first, lane);
    const int64_t b1 = warp_lower_bound(p.blk_row_grp, p.nb, p.n_rg, lane);
    unsigned long long lo = ~0ull, hi = 0ull;
    for (int64_t b = b0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < b1; b += (int64_t)gridDim.x * blockDim.x) {
        const unsigned long long g = (unsigned long long)__ldg(p.blk_col_grp + b);
        lo = g < lo ? g : lo;
        hi = g > hi ? g : hi;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long l2 = __shfl_xor_sync(kFullMask, lo, o), h2 = __shfl_xor_sync(kFullMask, hi, o);
        lo = l2 < lo ? l2 : lo;
        hi = h2 > hi ? h2 : hi;
    }
    if (lane == 0 && lo != ~0ull) {
        atomicMin(cg_range, lo);
        atomicMax(cg_range + 1, hi);
    }
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    return n;
}

// Gathered X panels, then 256 bytes for the column-group range of a
// row-group-range product.
template <int PW>
size_t gather_bytes(const spmm_boo_dev *A, int64_t batch, int64_t K) {
    return (size_t)batch * (size_t)A->n_cg * PW * (size_t)K * sizeof(float) + 256;
}

template <int NR, int PW, int NW, bool SPLIT>
int launch_tc(TcParams p, int64_t batch, void *ws, size_t ws_bytes, cudaStream_t s) {
    using Shape = TcShape<NR, PW, NW>;
    const int sms = sm_count();
    if (sms <= 0) return SPMM_ECUDA;
    const int64_t gather_rows = batch * p.n_cg * (PW / 4);
    if (gather_rows > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    const size_t xt_bytes = (size_t)gather_rows * (size_t)p.K * sizeof(float4);
    if (!ws || ws_bytes < xt_bytes + 256) return SPMM_EWORKSPACE;
    if ((uintptr_t)ws & 15) return SPMM_EALIGN;
    p.Xt = (const float4 *)ws;
    p.n_ft = p.K / kFeat;
    const int64_t n_rg = p.n_rg - p.rg_first;   // row groups of the range
    if (n_rg <= 0) return SPMM_OK;
    // chunks of consecutive row groups, small enough for ~16 tasks per worker
    const int64_t workers = (int64_t)sms * NW;
    int64_t c = n_rg / (16 * workers * p.n_ft * batch);
    c = c < 1 ? 1 : (c > 8 ? 8 : c);
    p.chunk_rgs = (int32_t)c;
    p.n_chunks = ceil_div(n_rg, c);
    p.n_tasks = p.n_chunks * p.n_ft * batch;
    if (p.n_tasks > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    const int64_t ctas = ceil_div(p.n_tasks, (int64_t)NW);
    const int grid = (int)(ctas < sms ? ctas : sms);
    auto kern = boo_tc_kernel<NR, PW, NW, SPLIT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Shape::kSmem);
    p.cg_range = nullptr;
    if (e == cudaSuccess && (p.rg_first != 0 || p.n_rg != p.n_rg_all)) {   // part of the row groups
        auto *range = reinterpret_cast<unsigned long long *>(static_cast<uint8_t *>(ws) + xt_bytes);
        e = cudaMemsetAsync(range, 0xFF, 8, s);
        if (e == cudaSuccess) e = cudaMemsetAsync(range + 1, 0, 8, s);
        if (e == cudaSuccess) {
            cg_range_kernel<<<(unsigned)(sms * 2), 256, 0, s>>>(p, range);
            e = cudaGetLastError();
        }
        p.cg_range = range;
    }
    if (e == cudaSuccess && gather_rows > 0) {
        boo_gather_kernel<PW><<<(unsigned)(batch * p.n_cg), 256, 0, s>>>(p);
        e = cudaGetLastError();
        if (e == cudaSuccess) note_product_launch();
    }
    if (e == cudaSuccess) {
        kern<<<grid, Shape::kThreads, Shape::kSmem, s>>>(p);
        e = cudaGetLastError();
        if (e == cudaSuccess) note_product_launch();
    }
    return e == cudaSuccess ? SPMM_OK : SPMM_ECUDA;
}

}  // namespace

bool tc_applicable(const spmm_boo_dev *A, int64_t K) {
    if (K < kFeat || K % kFeat || A->nb == 0 || A->n_cg <= 0) return false;
    if (A->n_rg > 0x7fffffffLL || A->nnz_c > 0x7fffffffLL) return false;
    return A->max_nr <= 64 && A->max_nc <= 64;
}

// Workspace of the tensor-core product (the gathered X panels), 0 when the
// CUDA-core product runs instead.
size_t boo_tc_workspace(const spmm_boo_dev *A, int64_t batch, int64_t K) {
    if (!tc_applicable(A, K)) return 0;
    if (A->max_nr <= 32 && A->max_nc <= 32) return gather_bytes<32>(A, batch, K);
    return gather_bytes<64>(A, batch, K);
}

// Tensor-core BOO product; SPMM_EUNSUPPORTED when the matrix or K does not
// fit the kernel (caller falls back to CUDA cores).  `ws`: the caller's
// scratch, 16-byte aligned, boo_tc_workspace() bytes (SPMM_EWORKSPACE when
// short).  `tf32_only`: one tf32 product per K step instead of the three-term
// split (SPMM_ENGINE_TENSOR_CORES_TF32, tf32 accuracy).  `status`: the call's status word (null: the process-wide
// g_tc_status); `wait_us` > 0 bounds the abortable waits to about that many
// microseconds instead of ~2 s; `flags` & SPMM_CFG_EXPIRE_FIRST_WAIT makes
// each worker's first wait expire (tests of the timeout path).
int boo_matmul_tc(const spmm_boo_dev *A, const float *X, float *Y, int64_t batch, int64_t K, int64_t rg_first,
                  int64_t rg_end, void *ws, size_t ws_bytes, int32_t *status, int32_t wait_us, int32_t flags,
                  bool tf32_only, const uint8_t *plan, cudaStream_t s) {
    if (!tc_applicable(A, K)) return SPMM_EUNSUPPORTED;
    if ((uintptr_t)X & 15) return SPMM_EUNSUPPORTED;  // 16-byte X loads
    if (!A->col_grp_ptr || !A->col_ids) return SPMM_EINVAL;
    TcParams p{};
    p.rows = A->rows;
    p.cols = A->cols;
    p.K = K;
    p.nb = A->nb;
    p.n_rg = rg_end;
    p.rg_first = rg_first;
    p.n_rg_all = A->n_rg;
    if (plan) {   // the matrix's plan: group table, and packed tiles when built for this panel width
        const PlanLayout L = plan_layout(A);
        p.rg_blk = reinterpret_cast<const int32_t *>(plan + L.rg_blk);
        if (L.packing) {
            p.packed = plan + L.packed;
            p.rg_slot = reinterpret_cast<const int32_t *>(plan + L.rg_slot);
            p.slots = reinterpret_cast<const int32_t *>(plan + L.slots);
            p.x_direct = reinterpret_cast<const int32_t *>(plan + L.cg_ident);
        }
    }
    p.rem_nnz = A->rem_nnz;
    p.tail_nnz = A->tail_nnz;
    p.row_grp_ptr = A->row_grp_ptr;
    p.row_ids = A->row_ids;
    p.col_grp_ptr = A->col_grp_ptr;
    p.col_ids = A->col_ids;
    p.blk_row_grp = A->blk_row_grp;
    p.blk_col_grp = A->blk_col_grp;
    p.blk_nz_ptr = A->blk_nz_ptr;
    p.blk_shift = A->blk_shift;
    p.nz_idx = A->nz_idx;
    p.nz_val = (const float *)A->nz_val;
    p.rem_indptr = A->rem_indptr;
    p.rem_col = A->rem_col_ind;
    p.rem_val = (const float *)A->rem_vals;
    p.tail_row = A->tail_row;
    p.tail_col = A->tail_col;
    p.tail_val = (const float *)A->tail_val;
    p.X = X;
    p.Y = Y;
    p.n_cg = A->n_cg;
    p.dense_nnz = kDenseNnz;
    if (status) {
        p.status = status;
    } else {
        void *g = nullptr;
        SPMM_CUDA_TRY(cudaGetSymbolAddress(&g, g_tc_status));
        p.status = (int *)g;
    }
    p.wait_cycles = wait_us > 0 ? (long long)wait_us * 2000 : kWaitCycles;   // ~2 GHz SM clock
    p.expire_probe = (flags & SPMM_CFG_EXPIRE_FIRST_WAIT) ? 1 : 0;
    if (A->max_nr <= 32 && A->max_nc <= 32)
        return tf32_only ? launch_tc<32, 32, 4, false>(p, batch, ws, ws_bytes, s)
                         : launch_tc<32, 32, 4, true>(p, batch, ws, ws_bytes, s);
    return tf32_only ? launch_tc<64, 64, 2, false>(p, batch, ws, ws_bytes, s)
                     : launch_tc<64, 64, 2, true>(p, batch, ws, ws_bytes, s);
}

}  // namespace spmm

extern "C" int spmm_tc_status(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, spmm::g_tc_status, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int z = 0;
        if (cudaMemcpyToSymbol(spmm::g_tc_status, &z, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}
