// k_scan_tc.cu -- the inverted-list scan on the tensor cores, for every metric
// (Cluster::search_into, AgentMemory/M3/src/cluster.cpp:229-274, driven by
// IVFIndex::search_nprobe, AgentMemory/M3/src/m3_index.cpp:368-483),
// list-centric like the SIMT scan (k_scan.cu): one work item is one list with
// up to 32 (k <= 32) or 16 (k <= 128) of the queries that probe it, so a list is
// normally streamed from HBM once per search batch.
//
// Two row formats: fp32 rows (the reference's storage, split into bf16 hi / lo
// on chip as below) and bf16 rows (half the bytes; the row is its own bf16 hi
// part, so only q is split: x . [q_hi | q_lo], two MMAs per 32 dims).
// Squared L2 is ranked by ||x||^2 - 2 <x, q> + ||q||^2 from the same dot
// product; the merge then rescores the answer's rows in the reference's own
// arithmetic (sum of (q_i - x_i)^2 in index order), since the expansion loses
// relative accuracy for rows very close to the query.
//
// Arithmetic.  <x, q> in fp32 accuracy from four bf16 MMAs per 32-dim chunk
// (tcgen05.mma kind::f16, K = 16, fp32 accumulation in TMEM): each fp32 value
// is split into two bf16 halves, x = x_hi + x_lo + e with x_hi = bf16(x),
// x_lo = bf16(x - x_hi) (round to nearest), |e| <= 2^-17 |x|, and likewise q.
//   x_hi . [q_hi | q_lo]   N = 2 nq_pad
//   x_lo . [q_hi | q_lo]   N = 2 nq_pad, into the same columns
// Every bf16 x bf16 product is exact in fp32; the column groups add up to
// (x_hi + x_lo)(q_hi + q_lo), within 2^-16 of each product x_i q_i.  The
// split warps convert each landed fp32 stage in place: a row's 128 bytes (32
// fp32 dims) become 64 bytes of x_hi and 64 bytes of x_lo, so the tensor core
// reads 16 KB per 128-row block and chunk (the fp32 data itself is never an
// MMA operand), and no second ring of correction tiles is needed.
//
// CTA (one per SM, 15 warps):
//   warp 0        producer: streams each queued item's rows by TMA (boxes of 32 dims x 128/64/32/16/8
//                 rows, SWIZZLE_128B, no multicast) through a ring of fp32 stages.
//   warp 1        MMA warp: keeps the loop state warp-uniform, one elected lane
//                 issues the MMAs and commits; it owns the TMEM allocation.
//   warps 2..9    split warps: per chunk, the bf16 query tile [q_hi | q_lo]; per
//                 stage, the in-place conversion of each row to [x_hi | x_lo].
//   warps 10..13  epilogue: TMEM -> scores -> a register top-k per query.
//   warp 14       scheduler: takes items from the global counter and queues
//                 their descriptors (list, rows, queries) up to NINFO ahead, so
//                 no role waits on that chain of global loads between items.
// Work order inside an item: passes of up to 256 / (2 nq_pad) row blocks of 128
// rows; inside a pass, chunk-pair-outer, block-inner: a 32 KB stage carries two
// consecutive 32-dim chunks of one block (so every stage is full but for a
// list's last, partial block), each block accumulating into its own 2 nq_pad
// TMEM columns, so the query tiles of a chunk pair serve every block of the pass.  TMEM is two halves of 256 columns: one pass accumulates while
// the epilogue drains the previous one.
// Every wait is bounded (mbar_wait); on an error the roles stop issuing, the
// issued copies and MMAs are drained, and TMEM is freed before the CTA leaves.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"
#include "topk.cuh"

namespace m3g {
namespace {

constexpr int TK = 32;                        // dims per chunk (128 B of fp32)
constexpr int TROWS = 128;                    // rows per block (MMA M)
constexpr int SCHK = 2;                       // chunks per stage (64 dims)
constexpr int CHK_BYTES = TROWS * TK * 4;     // 16 KB: one block's 32-dim chunk, fp32
constexpr int QMAX = 32;                      // queries per item (at most)
// the query tiles of a stage's two chunks: 64 rows [q_hi | q_lo] of 128 B, chunk j's
// 32 bf16 dims in bytes 64 j .. 64 j + 63 of each row
constexpr int QSLOT_BYTES = 2 * QMAX * 128;
constexpr int RING_BYTES = 192 * 1024;        // the stage ring: 6 x 32 KB fp32, 12 x 16 KB bf16
constexpr int NXS_MAX = 12;
constexpr int NQS = 2;                        // query chunk slots
constexpr int NSPLIT = 8;
constexpr int NEPI = 4;
constexpr int QHALF = 16;                     // queries per epilogue round through the score tile
constexpr int W_PROD = 0, W_MMA = 1, W_SPLIT0 = 2, W_EPI0 = W_SPLIT0 + NSPLIT;
constexpr int W_SCHED = W_EPI0 + NEPI;        // item scheduler warp
constexpr int NWARPS = W_SCHED + 1;
constexpr int NINFO = 4;                      // work items queued ahead of the roles
constexpr int NTHR = NWARPS * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr int HALF_COLS = 256;
constexpr int KMAX_TC = 128;
constexpr int EPI_BAR = 1;                    // named barrier of the epilogue warps

// Stage geometry of one row format: a stage is one 128-row block x 64 dims.
template <bool XB>
struct StageFmt {
    static constexpr int X_BYTES = XB ? TROWS * 128 : 2 * CHK_BYTES;  // 16 KB bf16, 32 KB fp32
    static constexpr int NXS = RING_BYTES / X_BYTES;                  // 12 / 6 stages
};
// Queries per item and register top-k width for a k limit.
template <int KW>
struct ItemFmt {
    static constexpr int QM = KW == 1 ? 32 : 16;  // queries per item
    static constexpr int QPW = QM / 4;            // queries per epilogue warp
};
static_assert(NSPLIT * 32 == SCHK * TROWS, "a split thread owns one row of one chunk of a stage");
static_assert(QSLOT_BYTES % 1024 == 0, "query tiles stay 1024-byte aligned");
static_assert(NSPLIT * 32 == QMAX * 8, "a split thread owns 16 bytes of a query chunk");

struct ItemTC {
    int32_t list;     // -1: no more items
    int32_t np;
    int32_t nrows;    // rows of this item
    int32_t tile_nt;  // > 0: a row tile (ScanItem)
    int64_t off;      // arena row of the item's first row
    int32_t row_begin, tile_out, tile_t, pad;
    int32_t q[QMAX];
    int32_t slot[QMAX];
};

struct LayoutTC {
    uint32_t x_off, q_off, sc_off, kb_off, info_off, bar_off, total;
};

__host__ __device__ constexpr LayoutTC make_layout_tc() {
    LayoutTC L{};
    uint32_t o = 0;
    L.x_off = o;
    o += RING_BYTES;
    L.q_off = o;
    o += NQS * QSLOT_BYTES;
    L.sc_off = o;
    o += QHALF * TROWS * 4;
    L.kb_off = o;
    o += QMAX * 32 * 8;
    L.info_off = o;
    o += NINFO * (uint32_t)sizeof(ItemTC);
    o = (o + 15u) & ~15u;
    L.bar_off = o;
    o += 3 * NXS_MAX * 8 + 64 * 8;
    L.total = o + 1024;  // slack for aligning the base to 1024 bytes
    return L;
}

static_assert(make_layout_tc().total <= 227u * 1024u, "shared memory layout too large");

// Ring position: index and phase parity, advanced one use at a time.
struct Ring {
    int i = 0;
    uint32_t ph = 0;
    uint32_t n = 0;  // uses so far
    __device__ __forceinline__ void next(int size) {
        ++n;
        if (++i == size) {
            i = 0;
            ph ^= 1u;
        }
    }
};

// bf16 pairs (round to nearest) of (a, b) in *hi and of the remainders
// (a - hi_a, b - hi_b) in *lo; element a in the low half.
__device__ __forceinline__ void bf16x2_split(float a, float b, uint32_t* hi, uint32_t* lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    *hi = *reinterpret_cast<const uint32_t*>(&h);
    *lo = *reinterpret_cast<const uint32_t*>(&l);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                       uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

__device__ __forceinline__ void sts64(uint32_t addr, uint32_t a, uint32_t b) {
    asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}

__device__ __forceinline__ float4 lds128f(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

// Item geometry shared by every role.
struct Geo {
    int np, nqp, nb, bpp, nrows;
    __device__ __forceinline__ explicit Geo(const ItemTC& inf) {
        np = inf.np;
        nrows = inf.nrows;
        nqp = np <= 16 ? 16 : 32;
        nb = (inf.nrows + TROWS - 1) / TROWS;
        bpp = HALF_COLS / (2 * nqp);
    }
};

// Row tiles: merges a (query, probe) pair's nt tile partial lists (at tile
// partials grp .. grp + nt - 1 of the tile region) by (score, row in the list)
// into the pair's own partial list `own`; list0 is the arena row of the list's
// row 0, buf the warp's 32-key buffer.  Called by the last tile to finish, after
// the atomic count showed every tile's list written.  Kept out of line: it is
// rare, and one copy serves every query slot of the epilogue.
template <int KW>
__device__ __noinline__ void merge_tile_lists(float* part_score, int64_t* part_row, int k,
                                              int64_t tile_base, int64_t grp, int nt, int64_t own,
                                              int64_t list0, unsigned long long* buf, int lane) {
    const float INF = __int_as_float(0x7f800000);
    __threadfence();
    RegTopKW<KW> m;
    for (int t = 0; t < nt; ++t) {
        const int64_t tb = (tile_base + grp + t) * (int64_t)k;
#pragma unroll
        for (int w = 0; w < KW; ++w) {
            const int e = 32 * w + lane;
            float sv = INF;
            int32_t rv = 0;
            if (e < k) {
                const int64_t r = __ldcg(part_row + tb + e);
                if (r >= 0) {
                    sv = __ldcg(part_score + tb + e);
                    rv = (int32_t)(r - list0);
                }
            }
            m.push(buf, k, sv, rv, lane);
        }
    }
    if (m.nbuf) m.flush(buf, k, lane);
    const int64_t ob = own * (int64_t)k;
#pragma unroll
    for (int w = 0; w < KW; ++w) {
        const int e = 32 * w + lane;
        if (e < k) {
            const unsigned long long t = m.top[w];
            const bool v = t != ~0ull;
            part_score[ob + e] = v ? key_float((uint32_t)(t >> 32)) : INF;
            part_row[ob + e] = v ? list0 + (int64_t)(uint32_t)(t & 0xffffffffu) : -1;
        }
    }
}

// XB: bf16 rows (else fp32); KW: register top-k width (k <= 32 KW).
template <bool XB, int KW>
__global__ void __launch_bounds__(NTHR, 1)
    list_scan_tc_kernel(const __grid_constant__ RowMaps maps, const ScanArgs a) {
    constexpr int X_BYTES = StageFmt<XB>::X_BYTES;
    constexpr int NXS = StageFmt<XB>::NXS;
    constexpr int QM = ItemFmt<KW>::QM;
    constexpr int QPW = ItemFmt<KW>::QPW;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const LayoutTC L = make_layout_tc();
    ItemTC* info = reinterpret_cast<ItemTC*>(smem + L.info_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* xfull = bars;               // NXS
    uint64_t* xempty = xfull + NXS;       // NXS
    uint64_t* xready = xempty + NXS;      // NXS: converted to bf16 by the split warps
    uint64_t* qfull = xready + NXS;       // NQS
    uint64_t* qempty = qfull + NQS;       // NQS
    uint64_t* infofull = qempty + NQS;    // NINFO
    uint64_t* infoempty = infofull + NINFO;  // NINFO
    uint64_t* accfull = infoempty + NINFO;   // 2
    uint64_t* accempty = accfull + 2;     // 2
    uint64_t* drain = accempty + 2;       // 1
    uint64_t* never = drain + 1;          // 1: the test hook's barrier, never arrived at
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(never + 1);
    float* sc = reinterpret_cast<float*>(smem + L.sc_off);
    unsigned long long* kbuf = reinterpret_cast<unsigned long long*>(smem + L.kb_off);
    const uint32_t x_u32 = smem_u32(smem + L.x_off);
    const uint32_t q_u32 = smem_u32(smem + L.q_off);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nchunks = (a.dpad + TK - 1) / TK;
    int* err = a.err;

    if (warp == W_MMA) tmem_alloc(tmem_slot, TMEM_COLS);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NXS; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], 1);
            mbar_init(&xready[s], NSPLIT);
        }
        for (int s = 0; s < NQS; ++s) {
            mbar_init(&qfull[s], NSPLIT);
            mbar_init(&qempty[s], 1);
        }
        for (int s = 0; s < NINFO; ++s) {
            mbar_init(&infofull[s], 1);
            mbar_init(&infoempty[s], 1 + NSPLIT + 1 + NEPI);  // producer, split, MMA, epilogue
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&accfull[s], 1);
            mbar_init(&accempty[s], NEPI);
        }
        mbar_init(drain, 1);
        mbar_init(never, 1);
        fence_mbar_init();
    }
    if (warp == W_PROD && lane == 0) {
        prefetch_tensormap(&maps.m128);
        prefetch_tensormap(&maps.m64);
        prefetch_tensormap(&maps.m32);
        prefetch_tensormap(&maps.m16);
        prefetch_tensormap(&maps.m8);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == W_PROD) {
        // ------------------------------ producer ------------------------------
        // The whole warp walks the schedule with warp-uniform values (so the
        // copy operands stay in uniform registers); the elected lane issues.
        const bool leader = elect_one();
        const uint32_t xbase = smem_u32(smem + L.x_off);
        Ring xr;
        bool ok = true;
        for (int it = 0; ok; ++it) {
            const int slot = it % NINFO;
            if (!__all_sync(0xffffffffu, mbar_wait(&infofull[slot], (it / NINFO) & 1, err))) break;
            const ItemTC* inf = &info[slot];
            if (inf->list < 0) break;
            const int np = inf->np, nrows = inf->nrows;
            const int64_t off = inf->off;
            const int nb = (nrows + TROWS - 1) / TROWS;
            const int bpp = HALF_COLS / (2 * (np <= 16 ? 16 : 32));
            for (int p0 = 0; p0 < nb && ok; p0 += bpp) {
                const int pb = min(bpp, nb - p0);
                for (int c = 0; c < nchunks && ok; c += SCHK) {
                    const int nch = min(SCHK, nchunks - c);
                    for (int b = 0; b < pb; ++b) {
                        if (xr.n >= (uint32_t)NXS &&
                            !__all_sync(0xffffffffu, mbar_wait(&xempty[xr.i], xr.ph ^ 1u, err))) {
                            ok = false;
                            break;
                        }
                        // the block's rows of each chunk as boxes of 128 / 64 / 32 / 16 / 8
                        // rows (rows past the list's end, up to the next multiple of 8, are
                        // read and masked later); chunk j of the stage at byte 16 KB * j
                        const int row0 = (p0 + b) * TROWS;
                        const int r8 = (min(TROWS, nrows - row0) + 7) & ~7;
                        const int y0 = (int)(off + row0);
                        uint64_t* bar = &xfull[xr.i];
                        // bf16 rows: one 64-dim box (128 B per row) covers the stage
                        const int nbox = XB ? 1 : nch;
                        if (leader) {
                            mbar_arrive_expect_tx(bar, (uint32_t)(nbox * r8 * 128));
                            for (int j = 0; j < nbox; ++j) {
                                const int x = (c + j) * TK;
                                const uint32_t dst = xbase + (uint32_t)xr.i * X_BYTES + j * CHK_BYTES;
                                if (r8 == 128) {
                                    tma_load_2d_u32(dst, &maps.m128, x, y0, bar);
                                } else {
                                    int r = 0;
                                    if (r8 - r >= 64) { tma_load_2d_u32(dst + r * 128, &maps.m64, x, y0 + r, bar); r += 64; }
                                    if (r8 - r >= 32) { tma_load_2d_u32(dst + r * 128, &maps.m32, x, y0 + r, bar); r += 32; }
                                    if (r8 - r >= 16) { tma_load_2d_u32(dst + r * 128, &maps.m16, x, y0 + r, bar); r += 16; }
                                    if (r8 - r >= 8) { tma_load_2d_u32(dst + r * 128, &maps.m8, x, y0 + r, bar); r += 8; }
                                }
                            }
                        }
                        __syncwarp();
                        xr.next(NXS);
                    }
                }
            }
            if (ok && leader) mbar_arrive(&infoempty[slot]);
            __syncwarp();
        }
        // no copy may still be landing when the CTA leaves
        if (leader) {
            for (uint32_t s = xr.n > (uint32_t)NXS ? xr.n - NXS : 0u; s < xr.n; ++s)
                mbar_drain(&xfull[s % NXS], (s / NXS) & 1u);
        }
        __syncwarp();
    } else if (warp == W_MMA) {
        // ------------------------------ MMA warp ------------------------------
        // The whole warp walks the schedule (waits, ring positions, descriptors:
        // all warp-uniform); the elected lane issues the MMAs and the commits.
        const bool leader = elect_one();
        // descriptor of slot 0 of each ring; a slot / K-step offset of b bytes
        // adds b >> 4 to the start-address field (shared addresses < 256 KB)
        const uint64_t dx0 = sw128_desc(x_u32);
        const uint64_t dq0 = sw128_desc(q_u32);
        Ring xr, qr;
        uint32_t pseq = 0;
        bool ok = true;
        for (int it = 0; ok; ++it) {
            const int slot = it % NINFO;
            if (!__all_sync(0xffffffffu, mbar_wait(&infofull[slot], (it / NINFO) & 1, err))) break;
            const ItemTC* inf = &info[slot];
            if (inf->list < 0) break;
            const Geo g(*inf);
            const uint32_t id_bf16 = tc_idesc_m128(2 * g.nqp, 1u);
            for (int p0 = 0; p0 < g.nb && ok; p0 += g.bpp) {
                const int pb = min(g.bpp, g.nb - p0);
                const int h = (int)(pseq & 1u);
                if (pseq >= 2 &&
                    !__all_sync(0xffffffffu, mbar_wait(&accempty[h], ((pseq >> 1) - 1) & 1u, err))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int c = 0; c < nchunks && ok; c += SCHK) {
                    const int nch = min(SCHK, nchunks - c);
                    if (!__all_sync(0xffffffffu, mbar_wait(&qfull[qr.i], qr.ph, err))) {
                        ok = false;
                        break;
                    }
                    const uint64_t dq = dq0 + (uint64_t)((qr.i * QSLOT_BYTES) >> 4);
                    for (int b = 0; b < pb; ++b) {
                        // fp32 rows wait for the split warps' conversion; bf16 rows are
                        // MMA operands as they land
                        uint64_t* ready = XB ? &xfull[xr.i] : &xready[xr.i];
                        if (!__all_sync(0xffffffffu, mbar_wait(ready, xr.ph, err))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (leader && XB) {
                            // row r of the stage: dims 0..63 as bf16 in its 128 B; K step
                            // k (16 dims, 32 B) meets the query tile's bytes 32 k .. 32 k + 31
                            const uint32_t d = tmem + (uint32_t)(h * HALF_COLS + b * 2 * g.nqp);
                            const uint64_t dx = dx0 + (uint64_t)((xr.i * X_BYTES) >> 4);
                            for (int k = 0; k < 2 * nch; ++k)
                                tc_mma_f16(d, dx + 2 * k, dq + 2 * k, id_bf16, (c | k) != 0);
                            tc_commit(&xempty[xr.i]);
                        } else if (leader) {
                            const uint32_t d = tmem + (uint32_t)(h * HALF_COLS + b * 2 * g.nqp);
                            for (int j = 0; j < nch; ++j) {
                                // chunk j's rows: x_hi in bytes 0..63, x_lo in 64..127
                                const uint64_t dx =
                                    dx0 + (uint64_t)((xr.i * X_BYTES + j * CHK_BYTES) >> 4);
                                const uint64_t dqj = dq + (uint64_t)(4 * j);  // 64 B per chunk
#pragma unroll
                                for (int k = 0; k < 2; ++k)  // K = 16 bf16 = 32 B per step
                                    tc_mma_f16(d, dx + 2 * k, dqj + 2 * k, id_bf16,
                                               ((c + j) | k) != 0);
#pragma unroll
                                for (int k = 0; k < 2; ++k)
                                    tc_mma_f16(d, dx + 4 + 2 * k, dqj + 2 * k, id_bf16, true);
                            }
                            tc_commit(&xempty[xr.i]);
                        }
                        __syncwarp();
                        xr.next(NXS);
                    }
                    if (!ok) break;
                    if (leader) tc_commit(&qempty[qr.i]);
                    __syncwarp();
                    qr.next(NQS);
                }
                if (!ok) break;
                if (leader) tc_commit(&accfull[h]);
                __syncwarp();
                ++pseq;
            }
            if (!ok) break;
            if (leader) mbar_arrive(&infoempty[slot]);
            __syncwarp();
        }
        // fires once every MMA issued above has completed
        if (leader) {
            tc_commit(drain);
            mbar_drain(drain, 0);
        }
        __syncwarp();
    } else if (warp < W_EPI0) {
        // ------------------------------ split warps ------------------------------
        const int s = threadIdx.x - W_SPLIT0 * 32;  // 0..255
        const int jh = s >> 7, r = s & (TROWS - 1);   // chunk of the stage, row of the block
        const int qn = s >> 3, qj = s & 7;           // query row, 16-byte column
        Ring xr, qr;
        for (int it = 0;; ++it) {
            const int slot = it % NINFO;
            const bool got = __all_sync(0xffffffffu, mbar_wait(&infofull[slot], (it / NINFO) & 1, err));
            if (!got) break;
            const ItemTC* inf = &info[slot];
            if (inf->list < 0) break;
            const Geo g(*inf);
            const int myq = qn < g.np ? inf->q[qn] : -1;
            const float* qrow = myq >= 0 ? a.Q + (int64_t)myq * a.dpad : nullptr;
            bool ok = true;
            // this thread's 16 bytes of the query tile of chunk c (global loads one
            // chunk ahead, so their latency hides behind the chunk's stages)
            auto qload = [&](int c) {
                const int d0 = c * TK + qj * 4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (qrow && d0 < a.dpad) v = __ldg(reinterpret_cast<const float4*>(qrow + d0));
                return v;
            };
            for (int p0 = 0; p0 < g.nb && ok; p0 += g.bpp) {
                const int pb = min(g.bpp, g.nb - p0);
                float4 qnext[SCHK];
#pragma unroll
                for (int j = 0; j < SCHK; ++j) qnext[j] = qload(j);
                for (int c = 0; c < nchunks && ok; c += SCHK) {
                    const int nch = min(SCHK, nchunks - c);
                    // query tiles of chunks c, c + 1: bf16 rows q_hi (qn) and q_lo (nqp + qn)
                    float4 qv[SCHK];
#pragma unroll
                    for (int j = 0; j < SCHK; ++j) {
                        qv[j] = qnext[j];
                        if (c + SCHK + j < nchunks) qnext[j] = qload(c + SCHK + j);
                    }
                    if (qr.n >= (uint32_t)NQS &&
                        !__all_sync(0xffffffffu, mbar_wait(&qempty[qr.i], qr.ph ^ 1u, err))) {
                        ok = false;
                        break;
                    }
                    if (qn < g.nqp) {
                        // dims 4 qj .. 4 qj + 3 of chunk j: 8 bytes in 16-byte column
                        // 4 j + qj / 2 of rows qn and nqp + qn (swizzled by row & 7, the
                        // same for both rows as nqp is a multiple of 8)
                        const uint32_t sw = (uint32_t)(qn & 7);
                        const uint32_t sl = q_u32 + (uint32_t)qr.i * QSLOT_BYTES;
#pragma unroll
                        for (int j = 0; j < SCHK; ++j) {
                            // (a chunk past the last holds zeros: qload gives them)
                            const uint32_t cb = ((((uint32_t)(4 * j + (qj >> 1))) ^ sw) << 4) +
                                                (uint32_t)(qj & 1) * 8;
                            uint32_t h0, h1, l0, l1;
                            bf16x2_split(qv[j].x, qv[j].y, &h0, &l0);
                            bf16x2_split(qv[j].z, qv[j].w, &h1, &l1);
                            sts64(sl + qn * 128 + cb, h0, h1);
                            sts64(sl + (g.nqp + qn) * 128 + cb, l0, l1);
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&qfull[qr.i]);
                    qr.next(NQS);
                    for (int b = 0; b < (XB ? 0 : pb); ++b) {
                        if (!__all_sync(0xffffffffu, mbar_wait(&xfull[xr.i], xr.ph, err))) {
                            ok = false;
                            break;
                        }
                        // warp-uniform: a warp's 32 rows share a chunk; rows past the
                        // block's last loaded one (a list's last block) hold stale bytes
                        // whose results the epilogue masks, so they are not converted
                        if (jh < nch && (p0 + b) * TROWS + (r & ~31) < g.nrows) {
                            // row r of chunk jh of the stage, in place: the 32 fp32 dims
                            // (16-byte columns 0..7) become x_hi in columns 0..3 and x_lo in
                            // columns 4..7, all swizzled by r & 7, the layout the MMA
                            // descriptors read.  The thread owns the row.
                            const uint32_t xb =
                                x_u32 + (uint32_t)xr.i * X_BYTES + (uint32_t)jh * CHK_BYTES + r * 128;
                            const uint32_t sw = (uint32_t)(r & 7);
                            float4 t[8];
#pragma unroll
                            for (int c8 = 0; c8 < 8; ++c8) t[c8] = lds128f(xb + (((uint32_t)c8 ^ sw) << 4));
#pragma unroll
                            for (int c4 = 0; c4 < 4; ++c4) {
                                uint32_t h[4], l[4];
                                bf16x2_split(t[2 * c4].x, t[2 * c4].y, &h[0], &l[0]);
                                bf16x2_split(t[2 * c4].z, t[2 * c4].w, &h[1], &l[1]);
                                bf16x2_split(t[2 * c4 + 1].x, t[2 * c4 + 1].y, &h[2], &l[2]);
                                bf16x2_split(t[2 * c4 + 1].z, t[2 * c4 + 1].w, &h[3], &l[3]);
                                sts128(xb + (((uint32_t)c4 ^ sw) << 4), h[0], h[1], h[2], h[3]);
                                sts128(xb + (((uint32_t)(4 + c4) ^ sw) << 4), l[0], l[1], l[2], l[3]);
                            }
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&xready[xr.i]);
                        xr.next(NXS);
                    }
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&infoempty[slot]);
        }
    } else if (warp == W_SCHED) {
        // ------------------------------ scheduler ------------------------------
        const bool leader = elect_one();
        const int nitems = *a.n_items;
        if (a.test_wait_ns) {
            // a bounded wait that runs out (its barrier never completes): the
            // timeout is recorded and the scan ends as if it had no items
            __all_sync(0xffffffffu, mbar_wait_for(never, 0, err, a.test_wait_ns));
            if (leader) {
                info[0].list = -1;
                mbar_arrive(&infofull[0]);
            }
            __syncwarp();
        }
        for (int it = 0; !a.test_wait_ns; ++it) {
            const int slot = it % NINFO;
            if (it >= NINFO &&
                !__all_sync(0xffffffffu,
                            mbar_wait(&infoempty[slot], ((it / NINFO) - 1) & 1, err)))
                break;
            ItemTC* inf = &info[slot];
            int item = 0;
            if (leader) item = atomicAdd(a.item_counter, 1);
            item = __shfl_sync(0xffffffffu, item, __ffs(__ballot_sync(0xffffffffu, leader)) - 1);
            if (item >= nitems) {
                if (leader) {
                    inf->list = -1;
                    mbar_arrive(&infofull[slot]);
                }
                break;
            }
            const ScanItem wi = a.items[item];
            const int np = wi.npairs;
            int nrows = 0;
            int64_t off = 0;
            if (wi.list >= 0) {
                const int len = a.list_len[wi.list];
                nrows = wi.nrows >= 0 ? min(wi.nrows, len - wi.row_begin) : len - wi.row_begin;
                off = a.list_off[wi.list] + wi.row_begin;
            }
            if (np < 1 || np > QM || nrows < 0 || wi.row_begin < 0 ||
                (wi.tile_nt > 0 && (!a.tile_cnt || wi.tile_out < 0 || wi.tile_t >= wi.tile_nt))) {
                if (leader) {
                    atomicCAS(err, 0, (int)kErrBadItem);
                    inf->list = -1;
                    mbar_arrive(&infofull[slot]);
                }
                break;
            }
            if (lane < np) {
                inf->q[lane] = a.pair_q[wi.pair_begin + lane];
                inf->slot[lane] = a.pair_slot[wi.pair_begin + lane];
            }
            if (leader) {
                inf->list = wi.list;
                inf->np = np;
                inf->nrows = nrows;
                inf->off = off;
                inf->tile_nt = wi.tile_nt;
                inf->row_begin = wi.row_begin;
                inf->tile_out = wi.tile_out;
                inf->tile_t = wi.tile_t;
            }
            __syncwarp();
            if (leader) mbar_arrive(&infofull[slot]);
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        // Two ways to spread an item over the four epilogue warps:
        //  * k > 32 and few queries (np <= QPW, "row split"): every warp takes the rows of its own
        //    TMEM lanes for every query, straight from its tcgen05.ld, and keeps a
        //    top-k per query over those rows; at the item's end the four lists of a
        //    query are merged by the warp that owns it (query j: warp j % 4);
        //  * more queries: warp ew keeps queries ew, ew + 4, ...; each block's scores
        //    pass through the score tile so that each warp reads all 128 rows.
        // Every decision that leads to a named barrier is taken by all four warps
        // together (named_bar_sync_or), so no barrier is ever left half-joined.
        const int ew = warp - W_EPI0;
        const int quarter = warp & 3;         // TMEM lanes 32*quarter ..
        const int trow = quarter * 32 + lane; // row of the block this thread drains
        const float INF = __int_as_float(0x7f800000);
        // the row split's list exchange: [warp][query][32 KW] keys over the score tile
        // and the key buffers (both idle by then), 16 KB
        unsigned long long* pub = reinterpret_cast<unsigned long long*>(smem + L.sc_off);
        static_assert(NEPI * QPW * 32 * KW * 8 <= QHALF * TROWS * 4 + QMAX * 32 * 8,
                      "the row split's list exchange fits the score tile and key buffers");
        static_assert(NEPI * QPW * 32 <= QMAX * 32, "the row split's key buffers fit");
        uint32_t pseq = 0;
        for (int it = 0;; ++it) {
            const int slot = it % NINFO;
            const bool got = __all_sync(0xffffffffu, mbar_wait(&infofull[slot], (it / NINFO) & 1, err));
            if (named_bar_sync_or(EPI_BAR, NEPI * 32, !got)) break;
            const ItemTC* inf = &info[slot];
            if (inf->list < 0) break;
            const Geo g(*inf);
            const int nrows = inf->nrows;
            const int64_t off = inf->off;
            // (measured: a gain for the 4-level top-k of k > 32, a loss for k <= 32,
            // whose 32-entry lists are cheap and whose tau tightens faster over all rows)
            const bool rsplit = KW > 1 && g.np <= QPW;
            // state j holds query (rsplit ? j : ew + NEPI j); rows scoring above a
            // query's bound cannot reach its answer (the bound is the k-th best score
            // of one of its lists already scanned)
            RegTopKW<KW> rt[QPW];
#pragma unroll
            for (int j = 0; j < QPW; ++j) {
                const int qi = rsplit ? j : ew + NEPI * j;
                if (qi < g.np && a.qbound) {
                    const uint32_t bk = ~a.qbound[inf->q[qi]];  // score key (0xffffffff: none)
                    if (bk != 0xffffffffu) rt[j].set_cap(((unsigned long long)bk << 32) | 0xffffffffull);
                }
            }
            bool ok = true;
            for (int p0 = 0; p0 < g.nb; p0 += g.bpp) {
                const int pb = min(g.bpp, g.nb - p0);
                const int h = (int)(pseq & 1u);
                // this thread's rows of the pass: tombstones and norms are loaded before
                // the accumulators are waited for, so their latency overlaps the MMAs
                constexpr int MAXB = HALF_COLS / 32;
                uint32_t livem = 0;
                float nb2v[MAXB];
                const bool need_n2 = a.metric == kL2 || (a.metric == kCosine && !a.normalized);
#pragma unroll
                for (int b = 0; b < MAXB; ++b) {
                    nb2v[b] = 0.f;
                    const int lrow = (p0 + b) * TROWS + trow;
                    if (b < pb && lrow < nrows) {
                        if (a.alive[off + lrow] != 0) livem |= 1u << b;
                        if (need_n2) nb2v[b] = a.rnorm2[off + lrow];
                    }
                }
                const bool acc = __all_sync(0xffffffffu, mbar_wait(&accfull[h], (pseq >> 1) & 1u, err));
                if (named_bar_sync_or(EPI_BAR, NEPI * 32, !acc)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int b = 0; b < pb; ++b) {
                    const int lrow = (p0 + b) * TROWS + trow;  // row in the list
                    const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) +
                                           (uint32_t)(h * HALF_COLS + b * 2 * g.nqp);
                    const bool live = (livem >> b) & 1u;
                    float nb2 = 0.f;
#pragma unroll
                    for (int bb = 0; bb < MAXB; ++bb)
                        if (bb == b) nb2 = nb2v[bb];
                    // columns [0, nqp): x q_hi; [nqp, 2 nqp): x q_lo
                    auto score_of = [&](uint32_t c0, uint32_t c1, int qi) {
                        const float dot = __uint_as_float(c0) + __uint_as_float(c1);
                        float s = INF;
                        if (live) {
                            if (a.metric == kIP) s = -dot;
                            else if (a.metric == kL2)  // ranking only; rescored at the merge
                                s = (nb2 + a.qnorm2[inf->q[qi]]) - 2.f * dot;
                            else if (a.normalized) s = 1.f - dot;
                            else {
                                const float na = a.qnorm2[inf->q[qi]];
                                s = (na == 0.f || nb2 == 0.f) ? 1.f : 1.f - dot / sqrtf(na * nb2);
                            }
                        }
                        return s;
                    };
                    if (rsplit) {
                        // this warp's 32 rows for every query, no score tile
                        uint32_t c0[QHALF], c1[QHALF];
                        tmem_ld16(taddr, c0);
                        tmem_ld16(taddr + g.nqp, c1);
                        if ((p0 + b) * TROWS + quarter * 32 < nrows) {  // warp-uniform
#pragma unroll
                            for (int j = 0; j < QPW; ++j)
                                if (j < g.np)
                                    rt[j].push(kbuf + (ew * QPW + j) * 32, a.k,
                                               score_of(c0[j], c1[j], j), lrow, lane);
                        }
                        continue;
                    }
                    // 16 queries per round: drained to the score tile, then pushed
#pragma unroll
                    for (int hq = 0; hq < QM / QHALF; ++hq) {
                        const int q0 = hq * QHALF;
                        if (q0 >= g.np) break;  // the same for every epilogue warp
                        uint32_t c0[QHALF], c1[QHALF];
                        tmem_ld16(taddr + q0, c0);
                        tmem_ld16(taddr + g.nqp + q0, c1);
#pragma unroll
                        for (int i = 0; i < QHALF; ++i)
                            if (q0 + i < g.np) sc[i * TROWS + trow] = score_of(c0[i], c1[i], q0 + i);
                        named_bar_sync(EPI_BAR, NEPI * 32);
#pragma unroll
                        for (int jj = 0; jj < QHALF / NEPI; ++jj) {
                            const int j = hq * (QHALF / NEPI) + jj;  // query ew + NEPI j
                            const int qi = ew + NEPI * j;
                            if (qi < g.np) {
                                unsigned long long* kb = kbuf + qi * 32;
                                const int rbase = (p0 + b) * TROWS;
#pragma unroll
                                for (int m = 0; m < TROWS / 32; ++m)
                                    if (rbase + 32 * m < nrows)
                                        rt[j].push(kb, a.k, sc[(qi - q0) * TROWS + 32 * m + lane],
                                                   rbase + 32 * m + lane, lane);
                            }
                        }
                        named_bar_sync(EPI_BAR, NEPI * 32);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&accempty[h]);
                ++pseq;
            }
            if (!ok) break;  // the same in every epilogue warp
            if (rsplit) {
                // drain the buffers, publish the lists of the queries other warps
                // own, and merge the three other lists of each owned query
#pragma unroll
                for (int j = 0; j < QPW; ++j)
                    if (j < g.np && rt[j].nbuf) rt[j].flush(kbuf + (ew * QPW + j) * 32, a.k, lane);
                named_bar_sync(EPI_BAR, NEPI * 32);
#pragma unroll
                for (int j = 0; j < QPW; ++j)
                    if (j < g.np && (j & (NEPI - 1)) != ew) {
#pragma unroll
                        for (int w = 0; w < KW; ++w)
                            pub[(ew * QPW + j) * 32 * KW + 32 * w + lane] = rt[j].top[w];
                    }
                named_bar_sync(EPI_BAR, NEPI * 32);
#pragma unroll
                for (int j = 0; j < QPW; ++j)
                    if (j < g.np && (j & (NEPI - 1)) == ew) {
#pragma unroll
                        for (int v = 0; v < NEPI; ++v)
                            if (v != ew) rt[j].merge_sorted(pub + (v * QPW + j) * 32 * KW, a.k, lane);
                    }
            }
            // the item's answers: top-k per (query, probe slot)
            uint32_t last_mask = 0;  // bit j: query slot j finished its pair's last tile
#pragma unroll
            for (int j = 0; j < QPW; ++j) {
                const int qi = rsplit ? j : ew + NEPI * j;
                const bool mine = rsplit ? (j < g.np && (j & (NEPI - 1)) == ew) : qi < g.np;
                if (mine) {
                    if (rt[j].nbuf) rt[j].flush(kbuf + qi * 32, a.k, lane);
                    // a full top-k bounds the query's final k-th score
                    const unsigned long long kth = rt[j].entry(a.k - 1);
                    if (a.qbound && lane == 0 && kth != ~0ull)
                        atomicMax(&a.qbound[inf->q[qi]], ~(uint32_t)(kth >> 32));
                    const int64_t own = (int64_t)inf->q[qi] * a.P + inf->slot[qi];
                    const int nt = inf->tile_nt;
                    // a row tile writes to its tile partial list
                    const int64_t grp = nt > 0 ? (int64_t)inf->tile_out + (int64_t)qi * nt : 0;
                    const int64_t base =
                        (nt > 0 ? a.tile_base + grp + inf->tile_t : own) * (int64_t)a.k;
#pragma unroll
                    for (int w = 0; w < KW; ++w) {
                        const int e = 32 * w + lane;
                        if (e < a.k) {
                            const unsigned long long t = rt[j].top[w];
                            const bool v = t != ~0ull;
                            a.part_score[base + e] = v ? key_float((uint32_t)(t >> 32)) : INF;
                            a.part_row[base + e] =
                                v ? off + (int64_t)(uint32_t)(t & 0xffffffffu) : -1;
                        }
                    }
                    if (nt > 0) {
                        // the pair's last tile to finish (counted after its list is out)
                        // merges the pair's nt tile lists below
                        __threadfence();
                        __syncwarp();
                        int done = 0;
                        if (lane == 0) done = atomicAdd(&a.tile_cnt[grp], 1);
                        if (__shfl_sync(0xffffffffu, done, 0) == nt - 1) last_mask |= 1u << j;
                    }
                }
            }
            // the exchange area and key buffers are reused by the next item
            if (rsplit) named_bar_sync(EPI_BAR, NEPI * 32);
            // Row tiles: the last tile of a pair merges the pair's tile lists into the
            // pair's own partial list.  Only this warp's key buffer is touched (the
            // row split's exchange is over, and the other warps start the next item
            // at a barrier of all four).
#pragma unroll 1
            for (int j = 0; j < QPW; ++j) {
                if (!((last_mask >> j) & 1u)) continue;
                const int qi = rsplit ? j : ew + NEPI * j;
                const int nt = inf->tile_nt;
                merge_tile_lists<KW>(a.part_score, a.part_row, a.k, a.tile_base,
                                     (int64_t)inf->tile_out + (int64_t)qi * nt, nt,
                                     (int64_t)inf->q[qi] * a.P + inf->slot[qi],
                                     off - inf->row_begin, kbuf + qi * 32, lane);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&infoempty[slot]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

bool scan_tc_supported(int metric, int k) {
    return metric >= kL2 && metric <= kCosine && k >= 1 && k <= KMAX_TC;
}

int scan_tc_gmax(int k) { return k <= 32 ? ItemFmt<1>::QM : ItemFmt<4>::QM; }

cudaError_t launch_list_scan_tc(const RowMaps& maps, const ScanArgs& a, bool bf16_rows, int grid,
                                cudaStream_t st) {
    if (!scan_tc_supported(a.metric, a.k) || (a.dpad & 3)) return cudaErrorInvalidValue;
    const LayoutTC L = make_layout_tc();
    auto go = [&](auto kern) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)L.total);
        if (e != cudaSuccess) return e;
        kern<<<grid, NTHR, L.total, st>>>(maps, a);
        return cudaGetLastError();
    };
    if (bf16_rows) return a.k <= 32 ? go(list_scan_tc_kernel<true, 1>) : go(list_scan_tc_kernel<true, 4>);
    return a.k <= 32 ? go(list_scan_tc_kernel<false, 1>) : go(list_scan_tc_kernel<false, 4>);
}

}  // namespace m3g
