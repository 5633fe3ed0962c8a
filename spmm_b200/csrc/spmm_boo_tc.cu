// spmm_boo_tc.cu -- Y = A*X for a float32 BOO matrix on the 5th-generation
// tensor cores (tcgen05, kind::tf32, three-term split for fp32 accuracy).
//
// The reference multiplies each BOO block on CUDA cores, one thread per
// (block row, feature) with the block's X rows staged in shared memory
// (torch_fast_spdmm/kernels/boo_kernel.cu:410-595).  Here a block is a small
// dense product instead: for the row group's feature tile of 128 columns,
//
//     Yt[f][r] += sum_c  Xt[f][c] * Ablk[r][c]        (Yt = Y^T, Xt = X^T)
//
// is one tcgen05.mma with M = 128 features, N = NR block rows, K = the block's
// columns in steps of 8.  Xt (the gathered X rows of the block's column group,
// 128 features x PW columns) is the A operand and lives in tensor memory; the
// densified block (NR x PW, zero-filled) is the B operand in 128-byte-swizzled
// K-major shared memory; the accumulator Yt lives in tensor memory for the
// whole row group.  fp32 accuracy comes from the split x = hi + lo with hi =
// x truncated to tf32: Xhi*Ahi + Xlo*Ahi + Xhi*Alo (the dropped lo*lo term is
// below 2^-20 |a||x|).
//
// One persistent CTA per SM, warp-specialised:
//   warp 0           one thread issues the MMAs and commits slot releases;
//   warp 1           block metadata (chunk search, block descriptors);
//                    (low warp numbers: the schedulers favour older warps,
//                    and these two sit on every block's critical path;
//                    warps 2-3 are idle so the warpgroups below start on a
//                    tensor-memory lane quadrant boundary)
//   warps 4-7        epilogue: tensor memory -> registers, CSR remainder and
//                    COO tail of each row (the reference's remainder and tail
//                    kernels, boo_kernel.cu:905-937, pbr_kernel.cu:976-1049),
//                    one coalesced store of every Y element;
//   warps 8..8+4NL   NL loader warpgroups; loader j owns X slot j in tensor
//                    memory and three A tiles in shared memory.  Per block it
//                    loads the used K steps of the block's X panel (16-byte
//                    loads from the gathered copy below), splits and stores
//                    them to tensor memory, while the next block's nonzeros
//                    are scattered into the next A tile.
// Before the product a gather pass copies X column group by column group into
// Xt[batch][group][4-column quad][feature] (float4 of 4 columns), so that a
// panel row is 8 coalesced 16-byte loads instead of 32 scattered 4-byte ones.
// Work is split into tasks (batch, chunk of consecutive row groups, feature
// tile -- innermost) dealt round-robin to the CTAs, so that the CTAs sweep the
// matrix together: the X rows they share and the blocks of a chunk (read once
// per feature tile) stay in L2.
//
// Every wait is bounded (clock-limited); on expiry the CTA raises an abort
// flag, every role leaves its loop, outstanding MMAs are drained, tensor
// memory is released and a status word readable through spmm_tc_status() is
// set.
#include <climits>

#include "ptx.cuh"
#include "spmm_common.cuh"

namespace spmm {

__device__ int g_tc_status;  // 0, or the first abort code of a tensor-core launch

namespace {

constexpr int kFeat = 128;           // features per task: MMA M, tensor-memory lanes
constexpr int kDescRing = 64;        // block descriptors in flight (metadata warp -> loaders)
// Chunks in flight (metadata warp -> epilogue).  A loader asks for the
// descriptor of its block i+2 before it hands block i to the MMA, so the
// metadata warp must be able to post every chunk up to 3*NL blocks past the
// oldest row group the epilogue still waits for, even when each chunk holds a
// single one-block row group: the ring must exceed 3*NL + 2 entries, or the
// epilogue -> MMA -> loader -> metadata-warp wait cycle closes.
constexpr int kChunkRing = 32;
constexpr int kATiles = 3;           // A tiles per loader warpgroup
constexpr int kMaxChunkRgs = 8;      // row groups per chunk
// Blocks with at least kDenseNnz nonzeros go through the tensor cores; the
// others (and the CSR remainder) are summed on CUDA cores by the epilogue.  An
// M = 128 MMA costs ~50 cycles whatever N is, so a 32 x 32 block needs a few
// dozen nonzeros before 3 MMAs per 8 used columns beat per-nonzero FMAs.
constexpr int kDenseNnz = 48;
constexpr int kListCap = 1024;       // epilogue: staged (row, column, value) entries per pass
constexpr int kSegs = 32;            // epilogue: segments (sparse blocks, remainder rows) per pass
constexpr int kNzPre = 4;            // nonzeros per loader thread fetched ahead
constexpr long long kWaitCycles = 1ll << 32;  // ~2 s at 2 GHz

// kSpecial: the block has a non-finite value in A or in a gathered X column;
// those products were left out of the MMA and the epilogue adds them on CUDA
// cores, so 0 * Inf never appears in rows that do not use the value.
enum : uint32_t { kFirst = 1, kLast = 2, kEnd = 4, kSpecial = 8 };

struct TcParams {
    int64_t rows, cols, K, nb, n_rg, rem_nnz, tail_nnz;
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
    int64_t n_cg;
};

struct BlockDesc {
    int32_t cg, k0, k1, rg, task, pad;
    uint32_t shift, flags;
};

struct ChunkInfo {
    int32_t task, rg0, rg1, end;
    uint32_t mask;                     // bit i: row group rg0 + i has tensor-core blocks
    int32_t bstart[kMaxChunkRgs + 1];  // first block of each row group
    uint8_t ndense[kMaxChunkRgs];      // tensor-core blocks of each row group
};

// Epilogue scratch: the row group's CUDA-core partial sums, one copy per
// summing warp (warp w adds entries w, w + P, ... for all 128 features, 4 per
// lane), and one pass of staged entries.
template <int NR>
struct alignas(16) EpiSmem {
    static constexpr int P = NR <= 32 ? 4 : 2;   // summing warps / partial copies
    float ys[P][NR][kFeat];
    int32_t lcol[kListCap];
    float lval[kListCap];
    uint8_t lrow[kListCap];
    int32_t soff[kSegs + 1];   // prefix of the segments' entry counts
    int32_t sbase[kSegs];      // first entry (block nonzero or remainder index)
    int32_t scb[kSegs];        // block: first column of its group in col_ids; row segment: -1
    uint32_t saux[kSegs];      // block: index shift; row segment: local row
};

struct SlotMeta {
    uint32_t kmask, flags;
    uint64_t bdesc;  // shared-memory descriptor of the block's A tile (hi part)
};

template <int PW, int NL>
struct alignas(16) TcCtl {
    uint64_t full[NL], empty[NL];
    uint64_t dfull[2], dempty[2];
    uint64_t descfull[kDescRing], descempty[kDescRing];
    uint64_t chunkfull[kChunkRing], chunkempty[kChunkRing];
    uint64_t fin;
    uint32_t kmask[NL][2];  // K steps (8 columns) with nonzeros, per staged block
    uint32_t aspecial[NL][2];
    BlockDesc desc[kDescRing];
    ChunkInfo chunk[kChunkRing];
    SlotMeta meta[NL];
    uint32_t dvalid[2], dspecial[2];
    uint32_t tmem_base;
    volatile int abort;
};

template <int NR, int PW, int NL>
struct TcShape {
    static constexpr int kTileBytes = NR * PW * 4;               // one of hi / lo
    static constexpr int kTilesBytes = NL * kATiles * 2 * kTileBytes;
    static constexpr int kThreads = 32 * (8 + 4 * NL);
    // dynamic shared memory: A tiles (1024-aligned base), epilogue scratch,
    // control block (mbarriers: 8-byte alignment), each offset 128-aligned
    static constexpr int kEpiOff = kTilesBytes;
    static constexpr int kCtlOff = (kEpiOff + (int)sizeof(EpiSmem<NR>) + 127) & ~127;
    static constexpr int kSmem = 1024 + kCtlOff + (int)sizeof(TcCtl<PW, NL>);
    static_assert(kTilesBytes % 1024 == 0 && kCtlOff % 128 == 0, "shared-memory carve-out alignment");
    static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
    static constexpr uint32_t kTmemCols = 512;
    static_assert(2 * NR + NL * 2 * PW <= (int)kTmemCols, "tensor memory budget");
    static_assert(NR % 16 == 0 && NR >= 16 && NR <= 256, "MMA N for M = 128");
    static_assert(PW % 32 == 0 && PW <= 64, "panel width");
    static_assert(kChunkRing > 3 * NL + 2, "chunk ring shallower than the loaders' lookahead");
};

// ---- bounded waits ------------------------------------------------------

__device__ __forceinline__ void raise_abort(volatile int *abort, int code) {
    *abort = 1;
    atomicCAS(&g_tc_status, 0, code);
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
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity, volatile int *abort, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 16; ++i)
            if (mbar_try_wait_sleep(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            raise_abort(abort, code);
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

// Byte offset of A(r, c) in an NR x PW tile stored K-major with the 128-byte
// swizzle: 32 columns (128 B) per row and atom of 8 rows, the 16-byte chunk
// index XORed with the row within the atom; PW = 64 uses two such atoms.
template <int NR>
__device__ __forceinline__ uint32_t a_offset(uint32_t r, uint32_t c) {
    const uint32_t cc = c & 31u;
    return (c >> 5) * (NR * 128u) + r * 128u + ((((cc >> 2) ^ r) & 7u) << 4) + ((cc & 3u) << 2);
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

// First index i in [0, n) with a[i] >= key (a ascending), by a 32-way search
// of the whole warp.
__device__ __forceinline__ int64_t warp_lower_bound(const int32_t *a, int64_t n, int64_t key, int lane) {
    int64_t lo = 0, hi = n;
    while (hi - lo > 32) {
        const int64_t step = (hi - lo + 31) / 32;
        const int64_t pi = lo + lane * step;
        const bool pred = pi < hi && (int64_t)__ldg(a + pi) < key;
        const int c = __popc(__ballot_sync(kFullMask, pred));
        if (c == 0) return lo;
        const int64_t nhi = lo + c * step;
        lo = lo + (c - 1) * step + 1;
        hi = nhi < hi ? nhi : hi;
    }
    const int64_t pi = lo + lane;
    const bool pred = pi < hi && (int64_t)__ldg(a + pi) < key;
    return lo + __popc(__ballot_sync(kFullMask, pred));
}

// ---- roles ------------------------------------------------------------------

template <int NR, int PW, int NL>
__device__ void meta_role(const TcParams &p, TcCtl<PW, NL> &ctl, int lane) {
    volatile int *abort = &ctl.abort;
    const unsigned lt_mask = (1u << lane) - 1u;
    int64_t q = 0;     // descriptors issued (tensor-core blocks)
    int64_t cidx = 0;  // chunks issued
    bool ok = true;
    for (int64_t task = blockIdx.x; task < p.n_tasks && ok; task += gridDim.x) {
        const int64_t chunk = (task / p.n_ft) % p.n_chunks;
        const int64_t rg0 = chunk * p.chunk_rgs;
        const int64_t rg1 = rg0 + p.chunk_rgs < p.n_rg ? rg0 + p.chunk_rgs : p.n_rg;
        const int nrg = (int)(rg1 - rg0);
        const int64_t bl = warp_lower_bound(p.blk_row_grp, p.nb, rg0, lane);
        // Pass 1: blocks and tensor-core blocks per row group of the chunk.
        // The epilogue gets the chunk before its descriptors, so it can drain
        // accumulators (and sum the CUDA-core part) while they flow.
        int call[kMaxChunkRgs], cden[kMaxChunkRgs];
#pragma unroll
        for (int k = 0; k < kMaxChunkRgs; ++k) call[k] = cden[k] = 0;
        for (int64_t b0 = bl;; b0 += 32) {
            const int64_t b = b0 + lane;
            const int64_t rgb = b < p.nb ? (int64_t)__ldg(p.blk_row_grp + b) : INT64_MAX;
            const bool valid = rgb < rg1;
            const bool dense =
                valid && __ldg(p.blk_nz_ptr + b + 1) - __ldg(p.blk_nz_ptr + b) >= p.dense_nnz;
#pragma unroll
            for (int k = 0; k < kMaxChunkRgs; ++k) {
                call[k] += __popc(__ballot_sync(kFullMask, valid && rgb == rg0 + k));
                cden[k] += __popc(__ballot_sync(kFullMask, dense && rgb == rg0 + k));
            }
            if (__ballot_sync(kFullMask, valid) != kFullMask) break;
        }
        ChunkInfo ci{};
        ci.task = (int32_t)task;
        ci.rg0 = (int32_t)rg0;
        ci.rg1 = (int32_t)rg1;
        ci.bstart[0] = (int32_t)bl;
#pragma unroll
        for (int k = 0; k < kMaxChunkRgs; ++k) {
            ci.bstart[k + 1] = ci.bstart[k] + call[k];
            ci.ndense[k] = (uint8_t)(cden[k] < 255 ? cden[k] : 255);
            if (cden[k]) ci.mask |= 1u << k;
        }
        if (lane == 0) {
            const int s = (int)(cidx % kChunkRing);
            ok = wait_phase(&ctl.chunkempty[s], (uint32_t)((cidx / kChunkRing) & 1) ^ 1u, abort, 2);
            if (ok) {
                ctl.chunk[s] = ci;
                mbar_arrive(&ctl.chunkfull[s]);
            }
        }
        ok = __shfl_sync(kFullMask, ok, 0);
        ++cidx;
        if (!ok) break;
        // Pass 2: a descriptor per tensor-core block, in block order, flagged
        // first / last among its row group's tensor-core blocks.
        int posted[kMaxChunkRgs];
#pragma unroll
        for (int k = 0; k < kMaxChunkRgs; ++k) posted[k] = 0;
        const int64_t bend = ci.bstart[nrg < kMaxChunkRgs ? nrg : kMaxChunkRgs];
        for (int64_t b0 = bl; b0 < bend && ok; b0 += 32) {
            const int64_t b = b0 + lane;
            const bool valid = b < bend;
            BlockDesc d{};
            bool dense = false;
            int k = 0;
            if (valid) {
                d.k0 = __ldg(p.blk_nz_ptr + b);
                d.k1 = __ldg(p.blk_nz_ptr + b + 1);
                dense = d.k1 - d.k0 >= p.dense_nnz;
                d.rg = __ldg(p.blk_row_grp + b);
                k = (int)(d.rg - rg0);
                d.cg = __ldg(p.blk_col_grp + b);
                d.shift = __ldg(p.blk_shift + b);
                d.task = (int32_t)task;
            }
            int before = 0, mine_posted = 0, mine_total = 0;
#pragma unroll
            for (int kk = 0; kk < kMaxChunkRgs; ++kk) {
                const unsigned m = __ballot_sync(kFullMask, dense && k == kk);
                if (k == kk) {
                    before = __popc(m & lt_mask);
                    mine_posted = posted[kk];
                    mine_total = cden[kk];
                }
                posted[kk] += __popc(m);
            }
            const unsigned dm = __ballot_sync(kFullMask, dense);
            bool w = true;
            if (dense) {
                d.flags = (mine_posted + before == 0 ? kFirst : 0u) |
                          (mine_posted + before + 1 == mine_total ? kLast : 0u);
                const int64_t qq = q + __popc(dm & lt_mask);
                const int s = (int)(qq % kDescRing);
                w = wait_phase(&ctl.descempty[s], (uint32_t)((qq / kDescRing) & 1) ^ 1u, abort, 1);
                if (w) {
                    ctl.desc[s] = d;
                    mbar_arrive(&ctl.descfull[s]);
                }
            }
            ok = __all_sync(kFullMask, w);
            q += __popc(dm);
        }
    }
    if (!ok) return;
    // End markers: one descriptor per loader warpgroup, one chunk.
    bool w = true;
    if (lane < NL) {
        const int64_t qq = q + lane;
        const int s = (int)(qq % kDescRing);
        w = wait_phase(&ctl.descempty[s], (uint32_t)((qq / kDescRing) & 1) ^ 1u, abort, 1);
        if (w) {
            BlockDesc d{};
            d.flags = kEnd;
            ctl.desc[s] = d;
            mbar_arrive(&ctl.descfull[s]);
        }
    }
    if (lane == 0) {
        const int s = (int)(cidx % kChunkRing);
        if (wait_phase(&ctl.chunkempty[s], (uint32_t)((cidx / kChunkRing) & 1) ^ 1u, abort, 2)) {
            ChunkInfo ci{};
            ci.end = 1;
            ctl.chunk[s] = ci;
            mbar_arrive(&ctl.chunkfull[s]);
        }
    }
    __syncwarp();
}

template <int NR, int PW, int NL>
__device__ void loader_role(const TcParams &p, TcCtl<PW, NL> &ctl, uint8_t *tiles, uint32_t tmem, int j, int lt) {
    using Shape = TcShape<NR, PW, NL>;
    constexpr int KS = PW / 8;  // K steps of a panel
    volatile int *abort = &ctl.abort;
    const uint32_t bar = 2 + j;
    const uint32_t lane_addr = (uint32_t)((lt & ~31) << 16);
    const uint32_t xslot = tmem + 2 * NR + (uint32_t)j * 2 * PW;
    uint8_t *my_tiles = tiles + (size_t)j * kATiles * 2 * Shape::kTileBytes;

    // Thread 0 waits, the warpgroup learns the (uniform) outcome at a barrier.
    auto wg_wait = [&](uint64_t *b, uint32_t parity, int code) -> bool {
        bool w = true;
        if (lt == 0) w = wait_phase(b, parity, abort, code);
        return bar_and(bar, 128, w);
    };
    // Reads descriptor number i of this warpgroup (uniform result).
    auto get_desc = [&](int64_t i, BlockDesc &d) -> bool {
        const int64_t qq = (int64_t)j + (int64_t)NL * i;
        const int s = (int)(qq % kDescRing);
        const bool w = wg_wait(&ctl.descfull[s], (uint32_t)((qq / kDescRing) & 1), 3);
        if (w) d = ctl.desc[s];
        return w;
    };
    auto release_desc = [&](int64_t i) {
        const int64_t qq = (int64_t)j + (int64_t)NL * i;
        mbar_arrive(&ctl.descempty[qq % kDescRing]);
    };

    // Stages block descriptor d into A tile `t` and mask buffer `cb`: zero
    // the tile, scatter hi/lo, OR the mask of K steps with nonzeros.
    // ipre/vpre hold this thread's first kNzPre nonzeros (loaded earlier).
    auto stage = [&](const BlockDesc &d, int t, int cb, const uint16_t (&ipre)[kNzPre], const float (&vpre)[kNzPre]) {
        uint8_t *hi = my_tiles + (size_t)t * 2 * Shape::kTileBytes;
        float4 *z = reinterpret_cast<float4 *>(hi);
        const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 2 * Shape::kTileBytes / 16 / 128; ++u) z[lt + 128 * u] = zero;
        if (lt == 0) {
            ctl.kmask[j][cb] = 0u;
            ctl.aspecial[j][cb] = 0u;
        }
        named_bar_sync(bar, 128);
        const uint32_t shift = d.shift, cm = (1u << shift) - 1u;
        uint32_t m = 0u;
        bool special = false;
        auto put = [&](uint32_t idx, float v) {
            const uint32_t r = idx >> shift, c = idx & cm;
            if (r < (uint32_t)NR && c < (uint32_t)PW) {
                const uint32_t off = a_offset<NR>(r, c);
                if (!finite(v)) {
                    special = true;
                    v = 0.f;
                }
                const float h = tf32_hi(v);
                *reinterpret_cast<float *>(hi + off) = h;
                *reinterpret_cast<float *>(hi + Shape::kTileBytes + off) = v - h;
                m |= 1u << (c >> 3);
            }
        };
        const int n = d.k1 - d.k0;
#pragma unroll
        for (int u = 0; u < kNzPre; ++u)
            if (lt + 128 * u < n) put(ipre[u], vpre[u]);
        for (int e = lt + 128 * kNzPre; e < n; e += 128) put(__ldg(p.nz_idx + d.k0 + e), __ldg(p.nz_val + d.k0 + e));
        m = __reduce_or_sync(kFullMask, m);
        if ((lt & 31) == 0 && m) atomicOr(&ctl.kmask[j][cb], m);
        if (__any_sync(kFullMask, special) && (lt & 31) == 0) ctl.aspecial[j][cb] = 1u;
    };
    auto prefetch = [&](const BlockDesc &d, uint16_t (&ipre)[kNzPre], float (&vpre)[kNzPre]) {
        const int n = d.k1 - d.k0;
#pragma unroll
        for (int u = 0; u < kNzPre; ++u) {
            const int e = lt + 128 * u;
            ipre[u] = e < n ? __ldg(p.nz_idx + d.k0 + e) : (uint16_t)0;
            vpre[u] = e < n ? __ldg(p.nz_val + d.k0 + e) : 0.f;
        }
    };

    // Software pipeline over this warpgroup's blocks i = 0, 1, ...: while
    // block i's panel loads are in flight, block i+1 (nonzeros fetched one
    // iteration earlier) is scattered into its A tile and block i+2's
    // nonzeros are fetched.
    BlockDesc cur{}, nxt{}, nx2{};
    uint16_t i1[kNzPre], i2[kNzPre];
    float v1[kNzPre], v2[kNzPre];
    if (!get_desc(0, cur)) return;
    if (!(cur.flags & kEnd)) {
        prefetch(cur, i1, v1);
        stage(cur, 0, 0, i1, v1);
    }
    named_bar_sync(bar, 128);
    if (lt == 0) release_desc(0);  // every thread has its copy
    nxt.flags = kEnd;
    if (!(cur.flags & kEnd)) {
        if (!get_desc(1, nxt)) return;
        if (!(nxt.flags & kEnd)) prefetch(nxt, i1, v1);
        named_bar_sync(bar, 128);
        if (lt == 0) release_desc(1);
    }

    for (int64_t i = 0;; ++i) {
        const int t = (int)(i % kATiles), cb = (int)(i & 1);
        if (cur.flags & kEnd) {
            const bool w = i == 0 || wg_wait(&ctl.empty[j], (uint32_t)((i - 1) & 1), 4);
            if (w && lt == 0) {
                ctl.meta[j] = SlotMeta{0u, kEnd, 0ull};
                mbar_arrive(&ctl.full[j]);
            }
            return;
        }
        // 1. load the panel of the current block: this thread's feature of
        // the group's columns, 4 columns per 16-byte load, used K steps only
        const uint32_t kmask = ctl.kmask[j][cb];
        const bool aspecial = ctl.aspecial[j][cb] != 0u;
        const int64_t task = cur.task;
        const int64_t ft = task % p.n_ft, bt = task / (p.n_chunks * p.n_ft);
        const float4 *xq = p.Xt + ((bt * p.n_cg + cur.cg) * (PW / 4)) * p.K + ft * kFeat + lt;
        float x[PW];
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (kmask & (1u << ks)) {
                a = __ldg(xq + (2 * ks) * p.K);
                b = __ldg(xq + (2 * ks + 1) * p.K);
            }
            x[ks * 8 + 0] = a.x; x[ks * 8 + 1] = a.y; x[ks * 8 + 2] = a.z; x[ks * 8 + 3] = a.w;
            x[ks * 8 + 4] = b.x; x[ks * 8 + 5] = b.y; x[ks * 8 + 6] = b.z; x[ks * 8 + 7] = b.w;
        }
        // 2. descriptor and nonzeros of block i+2
        const bool more = !(nxt.flags & kEnd);
        nx2.flags = kEnd;
        if (more) {
            if (!get_desc(i + 2, nx2)) return;
            if (!(nx2.flags & kEnd)) prefetch(nx2, i2, v2);
        }
        // 3. block i+1 into the next A tile
        if (more) stage(nxt, (int)((i + 1) % kATiles), (int)((i + 1) & 1), i1, v1);
        // 4. wait until the MMAs of this slot's previous block are done
        const bool w = i == 0 || wg_wait(&ctl.empty[j], (uint32_t)((i - 1) & 1), 4);
        if (!w) return;
        if (more && lt == 0) release_desc(i + 2);  // every thread has its copy
        tc_fence_after();
        // 5. split and store the panel: hi at xslot, lo at xslot + PW
        bool xspecial = false;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            if (kmask & (1u << ks)) {
                uint32_t h[8], l[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float v = x[ks * 8 + e];
                    if (!finite(v)) {
                        xspecial = true;
                        v = 0.f;
                    }
                    const float hv = tf32_hi(v);
                    h[e] = __float_as_uint(hv);
                    l[e] = __float_as_uint(v - hv);
                }
                tmem_st8(xslot + lane_addr + ks * 8, h);
                tmem_st8(xslot + lane_addr + PW + ks * 8, l);
            }
        }
        tmem_wait_st();
        tc_fence_before();
        fence_proxy_async_smem();
        const bool special = bar_or(bar, 128, xspecial) || aspecial;
        if (lt == 0) {
            const uint32_t tile = smem_u32(my_tiles + (size_t)t * 2 * Shape::kTileBytes);
            ctl.meta[j] = SlotMeta{kmask, cur.flags | (special ? kSpecial : 0u), b_desc_sw128(tile)};
            mbar_arrive(&ctl.full[j]);
        }
        cur = nxt;
        nxt = nx2;
#pragma unroll
        for (int u = 0; u < kNzPre; ++u) {
            i1[u] = i2[u];
            v1[u] = v2[u];
        }
    }
}

template <int NR, int PW, int NL>
__device__ void mma_role(TcCtl<PW, NL> &ctl, uint32_t tmem) {
    using Shape = TcShape<NR, PW, NL>;
    constexpr int KS = PW / 8;
    constexpr uint32_t idesc = idesc_tf32<NR>();
    constexpr uint64_t kLoDesc = Shape::kTileBytes >> 4;  // hi tile -> lo tile, descriptor units
    volatile int *abort = &ctl.abort;
    uint32_t dbuf = 0, du[2] = {0u, 0u};
    uint32_t started = 0, special = 0;
    // One thread issues; the tensor pipe takes an M = 128 MMA about every 50
    // cycles, so the loop keeps per-MMA work to an add and the instruction:
    // descriptors come precomputed and K-step offsets are constants.
    for (uint32_t q = 0;; ++q) {
        const uint32_t j = q % NL;
        if (!wait_phase(&ctl.full[j], (q / NL) & 1u, abort, 5)) break;
        tc_fence_after();
        const SlotMeta m = ctl.meta[j];
        if (m.flags & kEnd) break;
        if (m.flags & kFirst) {
            if (!wait_phase(&ctl.dempty[dbuf], (du[dbuf] & 1u) ^ 1u, abort, 6)) break;
            tc_fence_after();
            started = 0;
            special = 0;
        }
        special |= m.flags & kSpecial;
        const uint32_t d = tmem + dbuf * NR;
        const uint32_t xa = tmem + 2 * NR + j * 2 * PW;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            if (m.kmask & (1u << ks)) {
                const uint64_t bh = m.bdesc + (uint64_t)(((ks >> 2) * (NR * 128) + (ks & 3) * 32) >> 4);
                mma_tf32_ts(d, xa + ks * 8, bh, idesc, started);
                mma_tf32_ts(d, xa + PW + ks * 8, bh, idesc, 1u);
                mma_tf32_ts(d, xa + ks * 8, bh + kLoDesc, idesc, 1u);
                started = 1;
            }
        }
        mma_commit(&ctl.empty[j]);
        if (m.flags & kLast) {
            ctl.dvalid[dbuf] = started;
            ctl.dspecial[dbuf] = special;
            mbar_arrive(&ctl.dfull[dbuf]);
            mma_commit(&ctl.dfull[dbuf]);
            ++du[dbuf];
            dbuf ^= 1u;
        }
    }
    // drain every MMA issued above before tensor memory is released
    mma_commit(&ctl.fin);
    wait_phase(&ctl.fin, 0u, abort, 7);
}

// CUDA-core part of row group rg, summed into e.ys (thread et owns feature
// column et): the entries of its blocks with fewer than dense_nnz nonzeros,
// then its rows' CSR remainder (the reference's remainder kernel,
// boo_kernel.cu:905-937).  Segments (one per block or row) are listed by warp
// 0, their entries staged as (local row, column, value) by all 128 threads,
// then each thread sums them for its feature with 16 X loads in flight.
template <int NR>
__device__ __forceinline__ void epi_cuda_part(const TcParams &p, EpiSmem<NR> &e, int32_t bs, int32_t be,
                                              int32_t rbase, int32_t nr, const float *xb, int et) {
    const int nblk = be - bs;
    const int nseg = nblk + (p.rem_nnz ? nr : 0);
    for (int s0 = 0; s0 < nseg; s0 += kSegs) {
        if (et < 32) {
            const int sidx = s0 + et;
            int cnt = 0, base = 0, cb = -1;
            uint32_t aux = 0;
            if (sidx < nblk) {
                const int64_t b = bs + sidx;
                const int32_t k0 = __ldg(p.blk_nz_ptr + b), k1 = __ldg(p.blk_nz_ptr + b + 1);
                if (k1 - k0 < p.dense_nnz) {
                    cnt = k1 - k0;
                    base = k0;
                    cb = __ldg(p.col_grp_ptr + __ldg(p.blk_col_grp + b));
                    aux = __ldg(p.blk_shift + b);
                }
            } else if (sidx < nseg) {
                const int r = sidx - nblk;
                const int32_t row = __ldg(p.row_ids + rbase + r);
                base = __ldg(p.rem_indptr + row);
                cnt = __ldg(p.rem_indptr + row + 1) - base;
                aux = (uint32_t)r;
            }
            int incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(kFullMask, incl, o);
                if (et >= o) incl += n;
            }
            e.soff[et + 1] = incl;
            if (et == 0) e.soff[0] = 0;
            e.sbase[et] = base;
            e.scb[et] = cb;
            e.saux[et] = aux;
        }
        named_bar_sync(1, 128);
        const int total = e.soff[kSegs];
        for (int g0 = 0; g0 < total; g0 += kListCap) {
            const int ne = total - g0 < kListCap ? total - g0 : kListCap;
            for (int i = et; i < ne; i += 128) {
                const int g = g0 + i;
                int lo = 0, hi = kSegs - 1;
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (e.soff[mid] <= g) lo = mid; else hi = mid - 1;
                }
                const int kidx = e.sbase[lo] + (g - e.soff[lo]);
                uint32_t r;
                int32_t col;
                float v;
                if (e.scb[lo] >= 0) {
                    const uint32_t idx = __ldg(p.nz_idx + kidx), sh = e.saux[lo];
                    r = idx >> sh;
                    col = __ldg(p.col_ids + e.scb[lo] + (int32_t)(idx & ((1u << sh) - 1u)));
                    v = __ldg(p.nz_val + kidx);
                } else {
                    r = e.saux[lo];
                    col = __ldg(p.rem_col + kidx);
                    v = __ldg(p.rem_val + kidx);
                }
                e.lrow[i] = (uint8_t)(r < (uint32_t)NR ? r : 255u);
                e.lcol[i] = col;
                e.lval[i] = v;
            }
            named_bar_sync(1, 128);
            constexpr int P = EpiSmem<NR>::P;
            const int w = et >> 5, l4 = (et & 31) * 4;
            if (w < P) {
                // warp w: entries w, w + P, ...; lane: features 4l..4l+3
                const float4 *x4 = reinterpret_cast<const float4 *>(xb - et + l4);
                const int64_t k4 = p.K / 4;
                constexpr int U = 8;
                int i = w;
                for (; i + (U - 1) * P < ne; i += U * P) {
                    float4 x[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) x[u] = __ldg(x4 + (int64_t)e.lcol[i + u * P] * k4);
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const uint32_t r = e.lrow[i + u * P];
                        const float v = e.lval[i + u * P];
                        if (r < (uint32_t)NR) {
                            float4 *y = reinterpret_cast<float4 *>(&e.ys[w][r][l4]);
                            float4 t = *y;
                            t.x = fmaf(v, x[u].x, t.x);
                            t.y = fmaf(v, x[u].y, t.y);
                            t.z = fmaf(v, x[u].z, t.z);
                            t.w = fmaf(v, x[u].w, t.w);
                            *y = t;
                        }
                    }
                }
                for (; i < ne; i += P) {
                    const float4 x = __ldg(x4 + (int64_t)e.lcol[i] * k4);
                    const uint32_t r = e.lrow[i];
                    const float v = e.lval[i];
                    if (r < (uint32_t)NR) {
                        float4 *y = reinterpret_cast<float4 *>(&e.ys[w][r][l4]);
                        float4 t = *y;
                        t.x = fmaf(v, x.x, t.x);
                        t.y = fmaf(v, x.y, t.y);
                        t.z = fmaf(v, x.z, t.z);
                        t.w = fmaf(v, x.w, t.w);
                        *y = t;
                    }
                }
            }
            named_bar_sync(1, 128);  // the list is reused by the next pass
        }
        named_bar_sync(1, 128);      // the segment table is rewritten next
    }
}

// Rare contributions, summed into e.ys by each thread for its feature: the
// tensor-core block products left out for a non-finite operand (`special`),
// and the COO tail (the reference's tail kernel, pbr_kernel.cu:976-1049).
// Rolled loops, so the hot epilogue stays small for the instruction cache.
template <int NR>
__device__ __forceinline__ void epi_rare(const TcParams &p, EpiSmem<NR> &e, int32_t bs, int32_t be, int32_t rbase,
                                         int32_t nr, bool special, const float *xb, int et) {
    if (special) {
        for (int64_t b = bs; b < be; ++b) {
            const int32_t k0 = __ldg(p.blk_nz_ptr + b), k1 = __ldg(p.blk_nz_ptr + b + 1);
            if (k1 - k0 < p.dense_nnz) continue;
            const uint32_t shift = __ldg(p.blk_shift + b), cm = (1u << shift) - 1u;
            const int32_t cbase = __ldg(p.col_grp_ptr + __ldg(p.blk_col_grp + b));
            for (int32_t k = k0; k < k1; ++k) {
                const uint32_t idx = __ldg(p.nz_idx + k);
                const uint32_t r = idx >> shift;
                const float a = __ldg(p.nz_val + k);
                const float x = __ldg(xb + (int64_t)__ldg(p.col_ids + cbase + (int32_t)(idx & cm)) * p.K);
                if (r < (uint32_t)NR && (!finite(a) || !finite(x))) e.ys[0][r][et] = fmaf(a, x, e.ys[0][r][et]);
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
        float a = e.ys[0][r][et];
        for (int64_t k = lo; k < p.tail_nnz && __ldg(p.tail_row + k) == row; ++k)
            a = fmaf(__ldg(p.tail_val + k), __ldg(xb + (int64_t)__ldg(p.tail_col + k) * p.K), a);
        e.ys[0][r][et] = a;
    }
}

template <int NR>
__device__ __forceinline__ void zero_ys(EpiSmem<NR> &e, int et) {
    float4 *z = reinterpret_cast<float4 *>(&e.ys[0][0][0]);
    constexpr int n4 = EpiSmem<NR>::P * NR * kFeat / 4;
#pragma unroll 4
    for (int i = et; i < n4; i += 128) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

template <int NR, int PW, int NL>
__device__ void epilogue_role(const TcParams &p, TcCtl<PW, NL> &ctl, EpiSmem<NR> &e, uint32_t tmem, int et) {
    volatile int *abort = &ctl.abort;
    const uint32_t lane_addr = (uint32_t)((et & ~31) << 16);
    uint32_t dbuf = 0, du[2] = {0u, 0u};
    for (int64_t c = 0;; ++c) {
        const int s = (int)(c % kChunkRing);
        bool w = true;
        if (et == 0) w = wait_phase(&ctl.chunkfull[s], (uint32_t)((c / kChunkRing) & 1), abort, 8);
        if (!bar_and(1, 128, w)) return;
        const ChunkInfo ci = ctl.chunk[s];
        named_bar_sync(1, 128);
        if (et == 0) mbar_arrive(&ctl.chunkempty[s]);
        if (ci.end) return;
        const int64_t ft = ci.task % p.n_ft, bt = ci.task / (p.n_chunks * p.n_ft);
        const float *xb = p.X + bt * p.cols * p.K + ft * kFeat + et;
        float *yb = p.Y + bt * p.rows * p.K + ft * kFeat + et;
        for (int32_t rg = ci.rg0; rg < ci.rg1; ++rg) {
            const int k = rg - ci.rg0;
            const int32_t bs = ci.bstart[k], be = ci.bstart[k + 1];
            // row ids, one load round: lane l of every warp fetches rows
            // l, l + 32, ... and shuffles spread them
            constexpr int RH = (NR + 31) / 32;
            const int32_t rbase = __ldg(p.row_grp_ptr + rg);
            const int32_t nr = __ldg(p.row_grp_ptr + rg + 1) - rbase;
            int32_t myrow[RH];
#pragma unroll
            for (int h = 0; h < RH; ++h) {
                const int r = h * 32 + (et & 31);
                myrow[h] = r < nr && r < NR ? __ldg(p.row_ids + rbase + r) : -1;
            }
            // CUDA-core part first: it overlaps the MMAs of this row group
            const bool cuda_part = be - bs > (int32_t)ci.ndense[k] || p.rem_nnz;
            bool in_ys = cuda_part || p.tail_nnz;
            if (in_ys) {
                zero_ys<NR>(e, et);
                named_bar_sync(1, 128);
                if (cuda_part) epi_cuda_part<NR>(p, e, bs, be, rbase, nr, xb, et);
            }
            float acc[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] = 0.f;
            bool special = false;
            if ((ci.mask >> (uint32_t)k) & 1u) {
                w = true;
                if (et == 0) w = wait_phase(&ctl.dfull[dbuf], du[dbuf] & 1u, abort, 9);
                if (!bar_and(1, 128, w)) return;
                tc_fence_after();
                if (ctl.dvalid[dbuf]) {
#pragma unroll
                    for (int h = 0; h < NR / 16; ++h) {
                        uint32_t v[16];
                        tmem_ld16(tmem + dbuf * NR + lane_addr + h * 16, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int q = 0; q < 16; ++q) acc[h * 16 + q] = __uint_as_float(v[q]);
                    }
                }
                special = ctl.dspecial[dbuf] != 0u;
                tc_fence_before();
                mbar_arrive(&ctl.dempty[dbuf]);
                ++du[dbuf];
                dbuf ^= 1u;
            }
            if (special || p.tail_nnz) {
                if (!in_ys) {
                    zero_ys<NR>(e, et);
                    named_bar_sync(1, 128);
                    in_ys = true;
                }
                epi_rare<NR>(p, e, bs, be, rbase, nr, special, xb, et);
            }
            if (in_ys) named_bar_sync(1, 128);   // partials written by other warps
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const int32_t row = __shfl_sync(kFullMask, myrow[r / 32], r % 32);
                if (row >= 0) {
                    float y = acc[r];
                    if (in_ys) {
                        float c = e.ys[0][r][et];
#pragma unroll
                        for (int q = 1; q < EpiSmem<NR>::P; ++q) c += e.ys[q][r][et];
                        y = c + y;
                    }
                    __stcs(yb + (int64_t)row * p.K, y);
                }
            }
            if (in_ys) named_bar_sync(1, 128);   // partials are zeroed for the next group
        }
    }
}

template <int NR, int PW, int NL>
__global__ void __launch_bounds__(TcShape<NR, PW, NL>::kThreads, 1) boo_tc_kernel(const TcParams p) {
    using Shape = TcShape<NR, PW, NL>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *tiles = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    EpiSmem<NR> &epi = *reinterpret_cast<EpiSmem<NR> *>(tiles + Shape::kEpiOff);
    TcCtl<PW, NL> &ctl = *reinterpret_cast<TcCtl<PW, NL> *>(tiles + Shape::kCtlOff);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int j = 0; j < NL; ++j) {
            mbar_init(&ctl.full[j], 1);
            mbar_init(&ctl.empty[j], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl.dfull[b], 2);
            mbar_init(&ctl.dempty[b], 128);
        }
        for (int s = 0; s < kDescRing; ++s) {
            mbar_init(&ctl.descfull[s], 1);
            mbar_init(&ctl.descempty[s], 1);
        }
        for (int s = 0; s < kChunkRing; ++s) {
            mbar_init(&ctl.chunkfull[s], 1);
            mbar_init(&ctl.chunkempty[s], 1);
        }
        mbar_init(&ctl.fin, 1);
        ctl.abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&ctl.tmem_base, Shape::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl.tmem_base;

    if (warp == 0) {
        if (lane == 0) mma_role<NR, PW, NL>(ctl, tmem);
        __syncwarp();
    } else if (warp == 1) {
        meta_role<NR, PW, NL>(p, ctl, lane);
    } else if (warp >= 4 && warp < 8) {
        epilogue_role<NR, PW, NL>(p, ctl, epi, tmem, tid - 128);
    } else if (warp >= 8) {
        loader_role<NR, PW, NL>(p, ctl, tiles, tmem, (warp - 8) >> 2, tid - 256 - ((warp - 8) >> 2) * 128);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Shape::kTmemCols);
    }
}

// Gather pass: Xt[bt][g][q][f] = (X[bt][col 4q..4q+3 of group g][f]) as one
// float4, zeros past the group's size.  One CTA per (bt, g, q) row of Xt;
// reads and writes are coalesced over f.  HBM-bound streaming copy.
template <int PW>
__global__ void __launch_bounds__(128) boo_gather_kernel(const TcParams p) {
    constexpr int QW = PW / 4;
    const int64_t row = blockIdx.x;
    const int q = (int)(row % QW);
    const int64_t g = (row / QW) % p.n_cg, bt = row / (QW * p.n_cg);
    const int32_t cbase = __ldg(p.col_grp_ptr + g);
    const int32_t nc = __ldg(p.col_grp_ptr + g + 1) - cbase;
    const float *xr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = 4 * q + i;
        xr[i] = c < nc ? p.X + (bt * p.cols + __ldg(p.col_ids + cbase + c)) * p.K : nullptr;
    }
    float4 *out = const_cast<float4 *>(p.Xt) + row * p.K;
    for (int64_t f = threadIdx.x; f < p.K; f += 128) {
        float4 v;
        v.x = xr[0] ? __ldg(xr[0] + f) : 0.f;
        v.y = xr[1] ? __ldg(xr[1] + f) : 0.f;
        v.z = xr[2] ? __ldg(xr[2] + f) : 0.f;
        v.w = xr[3] ? __ldg(xr[3] + f) : 0.f;
        out[f] = v;
    }
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    return n;
}

template <int PW>
size_t gather_bytes(const spmm_boo_dev *A, int64_t batch, int64_t K) {
    return (size_t)batch * (size_t)A->n_cg * PW * (size_t)K * sizeof(float);
}

template <int NR, int PW, int NL>
int launch_tc(TcParams p, int64_t batch, void *ws, size_t ws_bytes, cudaStream_t s) {
    using Shape = TcShape<NR, PW, NL>;
    const int sms = sm_count();
    if (sms <= 0) return SPMM_ECUDA;
    const int64_t gather_rows = batch * p.n_cg * (PW / 4);
    if (gather_rows > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    const size_t need = (size_t)gather_rows * (size_t)p.K * sizeof(float4);
    void *own = nullptr;
    if (!ws || ws_bytes < need || ((uintptr_t)ws & 15)) {
        SPMM_CUDA_TRY(cudaMallocAsync(&own, need, s));
        ws = own;
    }
    p.Xt = (const float4 *)ws;
    p.n_ft = p.K / kFeat;
    // chunks of consecutive row groups: at least ~4 tasks per CTA, <= 8 groups
    int64_t c = p.n_rg / (4 * (int64_t)sms * p.n_ft * batch);
    c = c < 1 ? 1 : (c > 8 ? 8 : c);
    p.chunk_rgs = (int32_t)c;
    p.n_chunks = ceil_div(p.n_rg, c);
    p.n_tasks = p.n_chunks * p.n_ft * batch;
    if (p.n_tasks > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    const int grid = (int)(p.n_tasks < sms ? p.n_tasks : sms);
    auto kern = boo_tc_kernel<NR, PW, NL>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Shape::kSmem);
    if (e == cudaSuccess && gather_rows > 0) {
        boo_gather_kernel<PW><<<(unsigned)gather_rows, 128, 0, s>>>(p);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        kern<<<grid, Shape::kThreads, Shape::kSmem, s>>>(p);
        e = cudaGetLastError();
    }
    if (own) {
        const cudaError_t f = cudaFreeAsync(own, s);
        if (e == cudaSuccess) e = f;
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
// fit the kernel (caller falls back to CUDA cores).  `ws` (16-byte aligned,
// boo_tc_workspace() bytes) may be null: the gather buffer is then taken from
// the stream-ordered allocator and released after the launch.
int boo_matmul_tc(const spmm_boo_dev *A, const float *X, float *Y, int64_t batch, int64_t K, void *ws,
                  size_t ws_bytes, cudaStream_t s) {
    if (!tc_applicable(A, K)) return SPMM_EUNSUPPORTED;
    if ((uintptr_t)X & 15) return SPMM_EUNSUPPORTED;  // 16-byte X loads
    if (!A->col_grp_ptr || !A->col_ids) return SPMM_EINVAL;
    TcParams p{};
    p.rows = A->rows;
    p.cols = A->cols;
    p.K = K;
    p.nb = A->nb;
    p.n_rg = A->n_rg;
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
    if (A->max_nr <= 32 && A->max_nc <= 32) return launch_tc<32, 32, 4>(p, batch, ws, ws_bytes, s);
    return launch_tc<64, 64, 1>(p, batch, ws, ws_bytes, s);
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
