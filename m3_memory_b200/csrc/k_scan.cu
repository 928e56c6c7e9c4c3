// k_scan.cu -- the inverted-list scan with per-query top-k (Cluster::search_into,
// AgentMemory/M3/src/cluster.cpp:229-274, driven by IVFIndex::search_nprobe,
// AgentMemory/M3/src/m3_index.cpp:368-483), reorganised list-centric for the GPU.
//
// The reference walks queries one by one and, for each, the probed lists.  Here a
// search batch is turned around: the (query, probe) pairs are grouped by list, and
// each work item is one list with up to `gmax` of the queries that probe it, so a
// list is streamed from HBM once per item rather than once per query.
//
// Kernel shape (one persistent CTA per SM, warp-specialised):
//   warp 8      producer: takes items from a global counter, bulk-copies the
//               item's query rows into a double-buffered query area, and streams
//               the list's rows through a ring of shared-memory stages with 2-D TMA
//               (32 dims x up to 128 rows per stage, SWIZZLE_128B, no multicast).
//   warps 0..7  consumers: split K inside each stage -- warp w takes 16-byte
//               column slot w of every 32-dim stage, for rows lane + 32 m (m < 4),
//               keeping one fp32 FMA accumulator per (row, query); all eight warps
//               read each stage, so the whole ring beyond the current stage stays
//               in flight.  The eight partial sums are added in a fixed order,
//               turned into the unified score, masked by tombstones, and each warp
//               w < g folds the tile into the running top-k of query w (a register
//               bitonic sort + merge for k <= 32, an insertion list for larger k).
// Ordering: candidates are ranked by (score, probe slot, row in list), which is
// the reference's visiting order; scores differ from the reference's only by
// fp32 summation order.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace m3g {
namespace {

constexpr int KC = 32;          // dims per stage (128 bytes of fp32)
constexpr int RPL = 4;          // rows per lane
constexpr int TR = 32 * RPL;    // rows per tile
constexpr int NCW = 8;          // consumer warps
constexpr int NTHREADS = (NCW + 1) * 32;
constexpr int GMAX = 8;         // queries per item (upper bound of the runtime gmax)
constexpr int KMAX = 256;       // largest k the fused top-k keeps
constexpr int STAGE_BYTES = TR * KC * 4;
constexpr int MAX_STAGES = 12;
constexpr int MIN_STAGES = 3;
constexpr int PSTRIDE = GMAX + 1;  // partial-sum row stride (bank-conflict padding)
constexpr int SMEM_LIMIT = 227 * 1024;
static_assert(NCW == KC / 4, "each consumer warp owns one 16-byte column slot of a stage");

struct ItemInfo {
    int32_t list;      // -1: no more items
    int32_t pad0;
    int32_t npairs;
    int32_t nrows;
    int64_t off;       // first arena row of the list
    int32_t q[GMAX];
    int32_t slot[GMAX];
};

struct Layout {
    int nstage;
    int qstride;        // floats per query in shared memory (nchunks * 32, stored chunk-major)
    int gmax;
    uint32_t ring_off, q_off, part_off, sc_off, tks_off, tkr_off, info_off, bar_off, total;
};

__host__ __device__ inline int nchunks_of(int dpad) { return (dpad + KC - 1) / KC; }

__host__ __device__ inline Layout make_layout(int dpad, int gmax, int nstage) {
    Layout L;
    L.gmax = gmax;
    L.nstage = nstage;
    L.qstride = nchunks_of(dpad) * KC;
    uint32_t o = 0;
    L.ring_off = o;
    o += (uint32_t)nstage * STAGE_BYTES;
    L.q_off = o;
    o += 2u * (uint32_t)gmax * (uint32_t)L.qstride * 4u;
    L.part_off = o;
    o += (uint32_t)NCW * TR * PSTRIDE * 4u;
    L.sc_off = o;
    o += (uint32_t)GMAX * TR * 4u;
    L.tks_off = o;
    o += (uint32_t)GMAX * KMAX * 4u;
    L.tkr_off = o;
    o += (uint32_t)GMAX * KMAX * 4u;
    L.info_off = o;
    o += 2u * (uint32_t)sizeof(ItemInfo);
    o = (o + 15u) & ~15u;
    L.bar_off = o;
    o += (uint32_t)(2 * MAX_STAGES + 4) * 8u;
    L.total = o + 1024u;  // slack for aligning the ring to 1024 bytes
    return L;
}

__device__ __forceinline__ float4 lds128(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

// Producer side of the ring: waits until every stage it ever filled has landed
// (used when a launch ends early on an error, so no copy is left in flight).
__device__ void drain_stages(uint64_t* full, int nstage, uint32_t seq_end) {
    const uint32_t first = seq_end > (uint32_t)nstage ? seq_end - nstage : 0u;
    for (uint32_t s = first; s < seq_end; ++s) {
        uint64_t* b = &full[s % nstage];
        const uint32_t par = (s / nstage) & 1u;
        for (uint32_t i = 0; i < kWaitSpinLimit; ++i) {
            if (mbar_try_wait(b, par)) break;
            __nanosleep(256);
        }
    }
}

// One tile of up to 128 rows: every consumer warp walks all of the tile's
// stages; warp w takes the 16-byte column slot w of each 32-dim stage for rows
// lane + 32 m, so the eight warps share each stage and release it together.
// (stage, phase) is the consumer's ring position, advanced once per chunk.
// The item's queries sit chunk-major in shared memory at qbuf: chunk c of
// query i at byte (c * gmax + i) * 128.
template <int NQ, int RG, bool L2>
__device__ __forceinline__ void tile_chunks(const Layout& L, uint32_t ring, uint32_t qbuf,
                                            uint64_t* full, uint64_t* empty, int& stage,
                                            uint32_t& phase, int nchunks, int warp, int lane,
                                            float (&acc)[RPL][GMAX], int* err, bool& ok) {
#pragma unroll
    for (int r = 0; r < RPL; ++r)
#pragma unroll
        for (int i = 0; i < GMAX; ++i) acc[r][i] = 0.f;
    // rows lane + 32 m share (row & 7) = (lane & 7): the swizzled slot is the same
    const uint32_t off0 = ring + lane * 128 + ((warp ^ (lane & 7)) << 4);
    const uint32_t qstep = (uint32_t)L.gmax * KC * 4;
    uint32_t qa = qbuf + warp * 16;
    for (int c = 0; c < nchunks; ++c, qa += qstep) {
        bool got = ok && mbar_wait(&full[stage], phase, err);
        got = __all_sync(0xffffffffu, got);  // one decision per warp
        if (got) {
            const uint32_t base = off0 + (uint32_t)stage * STAGE_BYTES;
            float4 x[RG];
#pragma unroll
            for (int r = 0; r < RG; ++r) x[r] = lds128(base + r * 32 * 128);
            float4 qv[NQ];
#pragma unroll
            for (int qi = 0; qi < NQ; ++qi) qv[qi] = lds128(qa + qi * KC * 4);
            // component-major: consecutive FMAs update different accumulators
#define M3G_COMP(cx)                                                        \
    _Pragma("unroll") for (int r = 0; r < RG; ++r)                          \
        _Pragma("unroll") for (int qi = 0; qi < NQ; ++qi) {                 \
            if (L2) {                                                       \
                const float d = x[r].cx - qv[qi].cx;                        \
                acc[r][qi] = fmaf(d, d, acc[r][qi]);                        \
            } else {                                                        \
                acc[r][qi] = fmaf(x[r].cx, qv[qi].cx, acc[r][qi]);          \
            }                                                               \
        }
            M3G_COMP(x) M3G_COMP(y) M3G_COMP(z) M3G_COMP(w)
#undef M3G_COMP
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
        } else {
            // Leave the tile's barrier structure intact; the launch ends at the
            // next tile boundary with the error already recorded.
            ok = false;
        }
        if (++stage == L.nstage) {
            stage = 0;
            phase ^= 1u;
        }
    }
}

// g queries, rg active 32-row groups (rows past the tile's end cost nothing).
#define M3G_TILE_ARGS L, ring, qbuf, full, empty, stage, phase, nchunks, warp, lane, acc, err, ok
template <bool L2, int RG>
__device__ __forceinline__ void tile_dispatch_g(int g, const Layout& L, uint32_t ring,
                                                uint32_t qbuf, uint64_t* full, uint64_t* empty,
                                                int& stage, uint32_t& phase, int nchunks,
                                                int warp, int lane, float (&acc)[RPL][GMAX],
                                                int* err, bool& ok) {
#define M3G_TILE(n) \
    case n: tile_chunks<n, RG, L2>(M3G_TILE_ARGS); break;
    switch (g) {
        M3G_TILE(1) M3G_TILE(2) M3G_TILE(3) M3G_TILE(4) M3G_TILE(5) M3G_TILE(6) M3G_TILE(7)
        default: tile_chunks<8, RG, L2>(M3G_TILE_ARGS); break;
    }
#undef M3G_TILE
}

template <bool L2>
__device__ __forceinline__ void tile_dispatch(int g, int rg, const Layout& L, uint32_t ring,
                                              uint32_t qbuf, uint64_t* full, uint64_t* empty,
                                              int& stage, uint32_t& phase, int nchunks, int warp,
                                              int lane, float (&acc)[RPL][GMAX], int* err,
                                              bool& ok) {
    switch (rg) {
        case 1: tile_dispatch_g<L2, 1>(g, M3G_TILE_ARGS); break;
        case 2: tile_dispatch_g<L2, 2>(g, M3G_TILE_ARGS); break;
        case 3: tile_dispatch_g<L2, 3>(g, M3G_TILE_ARGS); break;
        default: tile_dispatch_g<L2, 4>(g, M3G_TILE_ARGS); break;
    }
}
#undef M3G_TILE_ARGS

// Folds up to 64 new (score, row) candidates (two per lane) into the sorted
// top-k kept in shared memory (tks ascending by (score, row); rows of this tile
// are larger than every row already held, so an equal score never displaces).
__device__ __forceinline__ void topk_fold(float* tks, int32_t* tkr, int& cnt, int k, float s0,
                                          int32_t row0, bool v0, float s1, int32_t row1, bool v1,
                                          int lane) {
    const float INF = __int_as_float(0x7f800000);
    float tau = cnt == k ? tks[k - 1] : INF;
    bool c0 = v0 && s0 < tau, c1 = v1 && s1 < tau;
    while (__any_sync(0xffffffffu, c0 || c1)) {
        // this lane's best candidate
        unsigned long long mine = ~0ull;
        if (c0) mine = ((unsigned long long)float_key(s0) << 32) | (uint32_t)row0;
        if (c1) {
            unsigned long long k1 = ((unsigned long long)float_key(s1) << 32) | (uint32_t)row1;
            if (k1 < mine) mine = k1;
        }
        unsigned long long best = mine;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            if (other < best) best = other;
        }
        const float bs = key_float((uint32_t)(best >> 32));
        const int32_t br = (int32_t)(best & 0xffffffffu);
        // insertion position: entries with score <= bs stay in front
        int pos = 0;
        for (int i = lane; i < cnt; i += 32) pos += tks[i] <= bs ? 1 : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) pos += __shfl_xor_sync(0xffffffffu, pos, o);
        const int last = cnt < k ? cnt : k - 1;  // entries [pos, last) move up by one
        float ms[KMAX / 32];
        int32_t mr[KMAX / 32];
#pragma unroll
        for (int m = 0; m < KMAX / 32; ++m) {
            const int i = pos + lane + 32 * m;
            if (i < last) {
                ms[m] = tks[i];
                mr[m] = tkr[i];
            }
        }
        __syncwarp();
#pragma unroll
        for (int m = 0; m < KMAX / 32; ++m) {
            const int i = pos + lane + 32 * m;
            if (i < last) {
                tks[i + 1] = ms[m];
                tkr[i + 1] = mr[m];
            }
        }
        if (lane == 0) {
            tks[pos] = bs;
            tkr[pos] = br;
        }
        __syncwarp();
        cnt = cnt < k ? cnt + 1 : k;
        if (c0 && s0 == bs && row0 == br) c0 = false;
        if (c1 && s1 == bs && row1 == br) c1 = false;
        tau = cnt == k ? tks[k - 1] : INF;
        c0 = c0 && s0 < tau;
        c1 = c1 && s1 < tau;
    }
}

__global__ void __launch_bounds__(NTHREADS, 1)
    list_scan_kernel(const __grid_constant__ RowMaps maps, const ScanArgs a, const Layout L) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* ring = smem + L.ring_off;
    float* qbase = reinterpret_cast<float*>(smem + L.q_off);
    float* part = reinterpret_cast<float*>(smem + L.part_off);
    float* sc = reinterpret_cast<float*>(smem + L.sc_off);
    float* tks_all = reinterpret_cast<float*>(smem + L.tks_off);
    int32_t* tkr_all = reinterpret_cast<int32_t*>(smem + L.tkr_off);
    ItemInfo* info = reinterpret_cast<ItemInfo*>(smem + L.info_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* empty = full + MAX_STAGES;
    uint64_t* qfull = empty + MAX_STAGES;
    uint64_t* qempty = qfull + 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nchunks = nchunks_of(a.dpad);
    const int qbuf_floats = L.gmax * L.qstride;

    // zero the query area once: its padding columns are never written again
    for (int i = threadIdx.x; i < 2 * qbuf_floats; i += NTHREADS) qbase[i] = 0.f;
    if (threadIdx.x == 0) {
        for (int s = 0; s < L.nstage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);  // every consumer warp reads every stage
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&qfull[b], 1);
            mbar_init(&qempty[b], NCW);
        }
        fence_mbar_init();
    }
    if (warp == NCW && lane == 0) {
        prefetch_tensormap(&maps.m128);
        prefetch_tensormap(&maps.m64);
        prefetch_tensormap(&maps.m32);
        prefetch_tensormap(&maps.m16);
        prefetch_tensormap(&maps.m8);
    }
    fence_proxy_async_smem();
    __syncthreads();

    if (warp == NCW) {
        // ------------------------------ producer ------------------------------
        uint32_t seq = 0;     // stages filled so far
        int pstage = 0;       // seq % nstage
        uint32_t pphase = 0;  // (seq / nstage) & 1
        const int nitems = *a.n_items;
        bool ok = true;
        int q_issued = 0;  // items whose query copies were issued
        for (int it = 0; ok; ++it) {
            const int qb = it & 1;
            if (it >= 2 && !mbar_wait(&qempty[qb], ((it >> 1) - 1) & 1, a.err)) {
                ok = false;
                break;
            }
            int item = 0;
            if (lane == 0) item = atomicAdd(a.item_counter, 1);
            item = __shfl_sync(0xffffffffu, item, 0);
            ItemInfo* inf = &info[qb];
            if (item >= nitems) {
                if (lane == 0) {
                    inf->list = -1;
                    mbar_arrive(&qfull[qb]);
                }
                break;
            }
            const ScanItem wi = a.items[item];
            const int np = wi.npairs;
            int nrows = 0;
            int64_t off = 0;
            if (wi.list >= 0) {
                nrows = a.list_len[wi.list];
                off = a.list_off[wi.list];
            }
            if (np < 1 || np > L.gmax || nrows < 0) {
                if (lane == 0) atomicCAS(a.err, 0, (int)kErrBadItem);
                if (lane == 0) {
                    inf->list = -1;
                    mbar_arrive(&qfull[qb]);
                }
                break;
            }
            int32_t myq = 0;
            if (lane < np) {
                myq = a.pair_q[wi.pair_begin + lane];
                inf->q[lane] = myq;
                inf->slot[lane] = a.pair_slot[wi.pair_begin + lane];
            }
            if (lane == 0) {
                inf->list = wi.list;
                inf->npairs = np;
                inf->nrows = nrows;
                inf->off = off;
            }
            __syncwarp();
            float* qdst = qbase + qb * qbuf_floats;
            if (lane == 0) mbar_arrive_expect_tx(&qfull[qb], (uint32_t)(np * a.dpad * 4));
            __syncwarp();
            // chunk-major: chunk c of query i to (c * gmax + i) * 32 floats
            for (int i = 0; i < np; ++i) {
                const int qrow = __shfl_sync(0xffffffffu, myq, i);
                for (int c = lane; c < nchunks; c += 32) {
                    const int n = min(KC, a.dpad - c * KC);
                    bulk_g2s(qdst + (c * L.gmax + i) * KC, a.Q + (int64_t)qrow * a.dpad + c * KC,
                             (uint32_t)(n * 4), &qfull[qb]);
                }
            }
            q_issued = it + 1;
            // stream the list: tiles of 128 rows, each as nchunks stages of 32 dims
            const int ntiles = (nrows + TR - 1) / TR;
            for (int t = 0; t < ntiles && ok; ++t) {
                const int rows_here = min(TR, nrows - t * TR);
                const int r8 = (rows_here + 7) & ~7;
                const int y0 = (int)(off + (int64_t)t * TR);
                // the tile's rows as boxes of 128 / 64 / 32 / 16 / 8 rows (rows past
                // the list's end, up to the next multiple of 8, are read and masked)
                for (int c = 0; c < nchunks; ++c) {
                    const int stage = pstage;
                    if (seq >= (uint32_t)L.nstage && !mbar_wait(&empty[stage], pphase ^ 1u, a.err)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0) {
                        unsigned char* dst = ring + (size_t)stage * STAGE_BYTES;
                        mbar_arrive_expect_tx(&full[stage], (uint32_t)(r8 * 128));
                        int r = 0;
                        const int x = c * KC;
                        if (r8 - r >= 128) { tma_load_2d(dst + r * 128, &maps.m128, x, y0 + r, &full[stage]); r += 128; }
                        if (r8 - r >= 64) { tma_load_2d(dst + r * 128, &maps.m64, x, y0 + r, &full[stage]); r += 64; }
                        if (r8 - r >= 32) { tma_load_2d(dst + r * 128, &maps.m32, x, y0 + r, &full[stage]); r += 32; }
                        if (r8 - r >= 16) { tma_load_2d(dst + r * 128, &maps.m16, x, y0 + r, &full[stage]); r += 16; }
                        if (r8 - r >= 8) { tma_load_2d(dst + r * 128, &maps.m8, x, y0 + r, &full[stage]); r += 8; }
                    }
                    ++seq;
                    if (++pstage == L.nstage) {
                        pstage = 0;
                        pphase ^= 1u;
                    }
                }
            }
        }
        if (!ok && lane == 0) {
            drain_stages(full, L.nstage, seq);
            if (q_issued > 0) {
                const int lit = q_issued - 1;
                for (uint32_t i = 0; i < kWaitSpinLimit; ++i) {
                    if (mbar_try_wait(&qfull[lit & 1], (lit >> 1) & 1)) break;
                    __nanosleep(256);
                }
            }
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    const int ctid = threadIdx.x;  // 0..255
    int stage = 0;        // ring position of the next stage to consume
    uint32_t phase = 0;
    const uint32_t ring_u32 = smem_u32(ring);
    float* tks = tks_all + warp * KMAX;
    int32_t* tkr = tkr_all + warp * KMAX;
    const float INF = __int_as_float(0x7f800000);
    for (int it = 0;; ++it) {
        const int qb = it & 1;
        bool ok = __all_sync(0xffffffffu, mbar_wait(&qfull[qb], (it >> 1) & 1, a.err));
        // every consumer warp takes the same exit decision here
        if (named_bar_sync_or(1, NCW * 32, !ok)) return;
        const ItemInfo* inf = &info[qb];
        const int list = inf->list;
        if (list < 0) return;
        const int g = inf->npairs, nrows = inf->nrows;
        const int64_t off = inf->off;
        const uint32_t qbuf = smem_u32(qbase + qb * qbuf_floats);
        int cnt = 0;  // this warp's query (warp < g): entries held in tks/tkr (k > 32)
        RegTopK rt;   // k <= 32: register top-k with its buffer in the tks area
        unsigned long long* kbuf = reinterpret_cast<unsigned long long*>(tks_all) + warp * 32;
        const bool reg_topk = a.k <= 32;
        const int ntiles = (nrows + TR - 1) / TR;
        for (int t = 0; t < ntiles; ++t) {
            float acc[RPL][GMAX];
            const int rows_here = min(TR, nrows - t * TR);
            const int rg = (rows_here + 31) >> 5;  // active 32-row groups
            if (a.metric == kL2)
                tile_dispatch<true>(g, rg, L, ring_u32, qbuf, full, empty, stage, phase, nchunks,
                                    warp, lane, acc, a.err, ok);
            else
                tile_dispatch<false>(g, rg, L, ring_u32, qbuf, full, empty, stage, phase, nchunks,
                                     warp, lane, acc, a.err, ok);
            float* pw = part + warp * TR * PSTRIDE;
#pragma unroll
            for (int r = 0; r < RPL; ++r)
#pragma unroll
                for (int qi = 0; qi < GMAX; ++qi)
                    if (qi < g && r < rg) pw[(lane + 32 * r) * PSTRIDE + qi] = acc[r][qi];
            // uniform stop if any warp's wait gave up during this tile
            if (named_bar_sync_or(1, NCW * 32, !ok)) return;
            for (int e = ctid; e < TR * g; e += NCW * 32) {
                const int r = e % TR, qi = e / TR;
                float s = INF;
                if (r < rows_here) {
                    float sum = 0.f;
#pragma unroll
                    for (int w = 0; w < NCW; ++w) sum += part[(w * TR + r) * PSTRIDE + qi];
                    const int64_t row = off + (int64_t)t * TR + r;
                    if (a.alive[row]) {
                        if (a.metric == kL2) s = sum;
                        else if (a.metric == kIP) s = -sum;
                        else if (a.normalized) s = 1.f - sum;
                        else {
                            const float na = a.qnorm2[inf->q[qi]], nb = a.rnorm2[row];
                            s = (na == 0.f || nb == 0.f) ? 1.f : 1.f - sum / sqrtf(na * nb);
                        }
                    }
                }
                sc[qi * TR + r] = s;
            }
            named_bar_sync(1, NCW * 32);
            if (warp < g) {
                const int rbase = t * TR;
#pragma unroll
                for (int h = 0; h < RPL; h += 2) {
                    const int ra = lane + 32 * h, rb = ra + 32;
                    const float s0 = sc[warp * TR + ra], s1 = sc[warp * TR + rb];
                    if (reg_topk) {
                        if (32 * h < rows_here) rt.push(kbuf, a.k, s0, rbase + ra, lane);
                        if (32 * (h + 1) < rows_here) rt.push(kbuf, a.k, s1, rbase + rb, lane);
                    } else {
                        topk_fold(tks, tkr, cnt, a.k, s0, rbase + ra, score_valid(s0), s1,
                                  rbase + rb, score_valid(s1), lane);
                    }
                }
            }
        }
        if (warp < g) {
            const int64_t base = ((int64_t)inf->q[warp] * a.P + inf->slot[warp]) * a.k;
            if (reg_topk) {
                if (rt.nbuf) rt.flush(kbuf, a.k, lane);
                if (lane < a.k) {
                    const bool v = rt.top != ~0ull;
                    a.part_score[base + lane] = v ? key_float((uint32_t)(rt.top >> 32)) : INF;
                    a.part_row[base + lane] =
                        v ? off + (int64_t)(uint32_t)(rt.top & 0xffffffffu) : -1;
                }
            } else {
                for (int j = lane; j < a.k; j += 32) {
                    a.part_score[base + j] = j < cnt ? tks[j] : INF;
                    a.part_row[base + j] = j < cnt ? off + tkr[j] : -1;
                }
            }
        }
        __syncwarp();
        // releases the query buffer and the item record to the producer
        if (lane == 0) mbar_arrive(&qempty[qb]);
    }
}

Layout choose_layout(int dpad, int* gmax_out) {
    for (int g = GMAX; g >= 1; g >>= 1) {
        for (int ns = MAX_STAGES; ns >= MIN_STAGES; --ns) {
            Layout L = make_layout(dpad, g, ns);
            if (L.total <= (uint32_t)SMEM_LIMIT) {
                *gmax_out = g;
                return L;
            }
        }
    }
    *gmax_out = 0;
    return make_layout(dpad, 1, MIN_STAGES);
}

}  // namespace

int scan_kmax() { return KMAX; }

int scan_gmax_for_dim(int dpad) {
    int g = 0;
    choose_layout(dpad, &g);
    return g;
}

cudaError_t launch_list_scan(const RowMaps& maps, const ScanArgs& a, int gmax, int grid,
                             cudaStream_t st) {
    int g = 0;
    Layout L = choose_layout(a.dpad, &g);
    if (g == 0 || gmax > g || a.k > KMAX) return cudaErrorInvalidValue;
    L = make_layout(a.dpad, gmax, L.nstage);
    cudaError_t e = cudaFuncSetAttribute(list_scan_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    list_scan_kernel<<<grid, NTHREADS, L.total, st>>>(maps, a, L);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Work list.
// ---------------------------------------------------------------------------
namespace {

// A pair enters the work list when its probe is a list id and, with skip_len,
// the list holds rows.
__device__ __forceinline__ bool pair_wanted(int l, int L, const int32_t* skip_len) {
    return l >= 0 && l < L && (!skip_len || skip_len[l] > 0);
}

__global__ void probe_hist_kernel(const int32_t* __restrict__ probes, int64_t n, int L,
                                  const int32_t* __restrict__ skip_len,
                                  int32_t* __restrict__ lcount) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int l = probes[i];
        if (pair_wanted(l, L, skip_len)) atomicAdd(&lcount[l], 1);
    }
}

constexpr int PLAN_THREADS = 1024;

__device__ __forceinline__ int items_of(int c, int gmax) { return (c + gmax - 1) / gmax; }


// Inclusive block-wide sum of one value per thread (PLAN_THREADS threads).
template <class T>
__device__ __forceinline__ T plan_block_scan(T v, T* wsum) {
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) wsum[w] = v;
    __syncthreads();
    if (w == 0) {
        T s = lane < PLAN_THREADS / 32 ? wsum[lane] : T(0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const T u = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += u;
        }
        if (lane < PLAN_THREADS / 32) wsum[lane] = s;
    }
    __syncthreads();
    return v + (w > 0 ? wsum[w - 1] : T(0));
}

// Lists probed by more query groups than this are not tiled: their groups
// already spread them over the SMs, and run side by side sharing its rows in L2.
constexpr int TILE_MAX_GROUPS = 2;

// Row tiles a list of len rows with c pairs asks for (1: not tiled).
__device__ __forceinline__ int tiles_of(int c, int len, int tile_rows, int gmax) {
    return (tile_rows > 0 && c > 0 && len > tile_rows && items_of(c, gmax) <= TILE_MAX_GROUPS)
               ? (len + tile_rows - 1) / tile_rows
               : 1;
}

// Tile partial lists a tiled list takes (c pairs x nt tiles); 0 when it is not
// tiled or could never fit the region alone.
__device__ __forceinline__ int64_t tile_cost(int c, int nt, int tile_cap) {
    const int64_t n = (int64_t)c * nt;
    return nt > 1 && n <= (int64_t)tile_cap ? n : 0;
}

// The work list is planned in three steps over the positions of list_order
// (longest list first): a grid gathers each position's pair count, rows and
// tile cost; one block scans those arrays into pair, item and tile offsets
// (deciding which lists are tiled); a grid writes every list's pair start and
// its items.  A list's pairs split into ceil(c / gmax) near-equal query groups;
// a tiled list repeats each group once per row tile.  A list is tiled when its
// tile partial lists fit the tile region after those of the lists before it in
// list_order that could fit on their own.
struct PlanArrays {
    int32_t* c;      // [L] pairs of the list at each position
    int32_t* len;    // [L] its rows (0 when not tiling)
    int32_t* cost;   // [L] tile partial lists it asks for, then the tiles it gets
    int32_t* pair0;  // [L] its first pair
    int32_t* item0;  // [L] its first item
    int32_t* tile0;  // [L] its first tile partial list (tiled lists)
};

__global__ void plan_gather_kernel(const int32_t* __restrict__ lcount,
                                   const int32_t* __restrict__ order,
                                   const int32_t* __restrict__ list_len, int L, int gmax,
                                   int tile_rows, int tile_cap, PlanArrays pa) {
    const bool tiled = tile_rows > 0 && list_len;
    for (int pos = blockIdx.x * blockDim.x + threadIdx.x; pos < L; pos += gridDim.x * blockDim.x) {
        const int l = order[pos];
        const int c = lcount[l];
        const int len = tiled ? list_len[l] : 0;
        pa.c[pos] = c;
        pa.len[pos] = len;
        pa.cost[pos] = (int32_t)tile_cost(c, tiles_of(c, len, tile_rows, gmax), tile_cap);
    }
}

// Inclusive sum over the lanes of a warp.
template <class T>
__device__ __forceinline__ T warp_incl_sum(T v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

// Exclusive offsets of the warps' totals (one value per warp in tot), in place.
template <class T>
__device__ __forceinline__ void plan_warp_offsets(T* tot, int warp, int lane) {
    __syncthreads();
    if (warp == 0) {
        const T v = lane < PLAN_THREADS / 32 ? tot[lane] : T(0);
        const T incl = warp_incl_sum(v, lane);
        if (lane < PLAN_THREADS / 32) tot[lane] = incl - v;
    }
    __syncthreads();
}

// One block.  Warp w takes rows of 32 consecutive positions (lane-contiguous, so
// every load is coalesced), PLAN_ROWS rows loaded together; prefixes come from
// warp scans, carried from row to row and offset by the scanned warp totals.
constexpr int PLAN_ROWS = 8;

__global__ void __launch_bounds__(PLAN_THREADS) plan_scan_kernel(int L, int gmax, int tile_rows,
                                                                 int tile_cap, PlanArrays pa,
                                                                 int32_t* __restrict__ n_items) {
    constexpr int NW = PLAN_THREADS / 32;
    __shared__ int32_t wp[NW], wi[NW];
    __shared__ int64_t wt[NW];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rows = (L + 32 * NW - 1) / (32 * NW);  // rows per warp
    const int base = warp * rows * 32;
    auto pos_of = [&](int r) { return base + r * 32 + lane; };
    // pass 1: the warp's pair and tile-cost totals
    int32_t np = 0;
    int64_t tc = 0;
    for (int r0 = 0; r0 < rows; r0 += PLAN_ROWS) {
        int32_t cv[PLAN_ROWS], kv[PLAN_ROWS];
#pragma unroll
        for (int u = 0; u < PLAN_ROWS; ++u) {
            const int p = pos_of(r0 + u);
            const bool in = r0 + u < rows && p < L;
            cv[u] = in ? pa.c[p] : 0;
            kv[u] = in ? pa.cost[p] : 0;
        }
#pragma unroll
        for (int u = 0; u < PLAN_ROWS; ++u) {
            np += cv[u];
            tc += kv[u];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        np += __shfl_xor_sync(0xffffffffu, np, o);
        tc += __shfl_xor_sync(0xffffffffu, tc, o);
    }
    if (lane == 0) {
        wp[warp] = np;
        wt[warp] = tc;
    }
    plan_warp_offsets(wp, warp, lane);
    plan_warp_offsets(wt, warp, lane);
    // pass 2: pair and tile offsets, the tiling decision, the item counts
    int32_t pcar = wp[warp];
    int64_t tcar = wt[warp];
    int32_t ni = 0;
    for (int r0 = 0; r0 < rows; r0 += PLAN_ROWS) {
        int32_t cv[PLAN_ROWS], kv[PLAN_ROWS], lv[PLAN_ROWS];
#pragma unroll
        for (int u = 0; u < PLAN_ROWS; ++u) {
            const int p = pos_of(r0 + u);
            const bool in = r0 + u < rows && p < L;
            cv[u] = in ? pa.c[p] : 0;
            kv[u] = in ? pa.cost[p] : 0;
            lv[u] = in ? pa.len[p] : 0;
        }
#pragma unroll
        for (int u = 0; u < PLAN_ROWS; ++u) {
            const int p = pos_of(r0 + u);
            const bool in = r0 + u < rows && p < L;
            const int32_t pin = warp_incl_sum(cv[u], lane);
            const int64_t tin = warp_incl_sum((int64_t)kv[u], lane);
            const int64_t tend = tcar + tin;  // tile lists up to and including this list
            const bool taken = kv[u] > 0 && tend <= (int64_t)tile_cap;
            const int nt = taken ? tiles_of(cv[u], lv[u], tile_rows, gmax) : 1;
            if (in) {
                pa.pair0[p] = pcar + pin - cv[u];
                pa.tile0[p] = taken ? (int32_t)(tend - kv[u]) : 0;
                pa.cost[p] = nt;
            }
            ni += items_of(cv[u], gmax) * nt;
            pcar += __shfl_sync(0xffffffffu, pin, 31);
            tcar += __shfl_sync(0xffffffffu, tin, 31);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ni += __shfl_xor_sync(0xffffffffu, ni, o);
    if (lane == 0) wi[warp] = ni;
    __syncthreads();
    if (threadIdx.x == 0) {
        int32_t total = 0;
        for (int w = 0; w < NW; ++w) total += wi[w];
        *n_items = total;
    }
    plan_warp_offsets(wi, warp, lane);
    // pass 3: item offsets
    int32_t icar = wi[warp];
    for (int r0 = 0; r0 < rows; r0 += PLAN_ROWS) {
        int32_t cv[PLAN_ROWS], nv[PLAN_ROWS];
#pragma unroll
        for (int u = 0; u < PLAN_ROWS; ++u) {
            const int p = pos_of(r0 + u);
            const bool in = r0 + u < rows && p < L;
            cv[u] = in ? pa.c[p] : 0;
            nv[u] = in ? pa.cost[p] : 1;
        }
#pragma unroll
        for (int u = 0; u < PLAN_ROWS; ++u) {
            const int p = pos_of(r0 + u);
            const int32_t v = items_of(cv[u], gmax) * nv[u];
            const int32_t inc = warp_incl_sum(v, lane);
            if (r0 + u < rows && p < L) pa.item0[p] = icar + inc - v;
            icar += __shfl_sync(0xffffffffu, inc, 31);
        }
    }
}

__global__ void plan_place_kernel(const int32_t* __restrict__ order, int L, int gmax,
                                  int tile_rows, PlanArrays pa, int32_t* __restrict__ lstart,
                                  ScanItem* __restrict__ items) {
    for (int pos = blockIdx.x * blockDim.x + threadIdx.x; pos < L; pos += gridDim.x * blockDim.x) {
        const int l = order[pos];
        const int c = pa.c[pos];
        const int pbase = pa.pair0[pos];
        lstart[l] = pbase;
        if (c <= 0) continue;
        const int n = items_of(c, gmax);
        const int nt = pa.cost[pos];
        const int ibase = pa.item0[pos];
        // tile-major: the query groups of one tile are neighbours in the work list,
        // so they run at the same time and share the tile's rows in L2
        int pb = pbase;
        for (int j = 0; j < n; ++j) {
            const int sz = c / n + (j < c % n ? 1 : 0);
            if (nt > 1) {
                const int len = pa.len[pos];
                const int32_t grp0 = pa.tile0[pos] + (pb - pbase) * nt;
                for (int r = 0; r < nt; ++r)
                    items[ibase + r * n + j] = ScanItem{
                        l, pb, sz, r * tile_rows, min(tile_rows, len - r * tile_rows), grp0, r, nt};
            } else {
                items[ibase + j] = ScanItem{l, pb, sz, 0, -1, -1, 0, 0};
            }
            pb += sz;
        }
    }
}

__global__ void pair_scatter_kernel(const int32_t* __restrict__ probes, int nq, int P, int L,
                                    const int32_t* __restrict__ skip_len,
                                    const int32_t* __restrict__ lstart,
                                    const int32_t* __restrict__ lcount,
                                    int32_t* __restrict__ lcursor, int32_t* __restrict__ pair_q,
                                    int32_t* __restrict__ pair_slot) {
    const int64_t n = (int64_t)nq * P;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int l = probes[i];
        if (!pair_wanted(l, L, skip_len)) continue;
        const int c = atomicAdd(&lcursor[l], 1);
        if (c >= lcount[l]) continue;  // never past the list's counted range
        pair_q[lstart[l] + c] = (int32_t)(i / P);
        pair_slot[lstart[l] + c] = (int32_t)(i % P);
    }
}

}  // namespace

cudaError_t launch_build_worklist(const int32_t* probes, int nq, int P, int L,
                                  const int32_t* list_order, int gmax, int32_t* lcount,
                                  int32_t* lstart, int32_t* lcursor, ScanItem* items,
                                  int32_t* n_items, int32_t* pair_q, int32_t* pair_slot,
                                  int32_t* plan, cudaStream_t st, const int32_t* skip_len,
                                  const int32_t* list_len, int tile_rows, int tile_cap) {
    if (tile_rows < 0 || tile_rows % 128 || tile_cap < 0 || (tile_rows > 0 && !list_len) ||
        (L > 0 && !plan))
        return cudaErrorInvalidValue;
    cudaError_t e;
    if ((e = cudaMemsetAsync(lcount, 0, sizeof(int32_t) * (size_t)L, st)) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(lcursor, 0, sizeof(int32_t) * (size_t)L, st)) != cudaSuccess) return e;
    const int64_t n = (int64_t)nq * P;
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
    if (n > 0) probe_hist_kernel<<<blocks, 256, 0, st>>>(probes, n, L, skip_len, lcount);
    if (L > 0) {
        const PlanArrays pa{plan, plan + L, plan + 2 * (size_t)L, plan + 3 * (size_t)L,
                            plan + 4 * (size_t)L, plan + 5 * (size_t)L};
        const int pg = (int)std::min<int64_t>((L + 255) / 256, 1184);
        plan_gather_kernel<<<pg, 256, 0, st>>>(lcount, list_order, list_len, L, gmax, tile_rows,
                                               tile_cap, pa);
        plan_scan_kernel<<<1, PLAN_THREADS, 0, st>>>(L, gmax, tile_rows, tile_cap, pa, n_items);
        plan_place_kernel<<<pg, 256, 0, st>>>(list_order, L, gmax, tile_rows, pa, lstart, items);
    } else if ((e = cudaMemsetAsync(n_items, 0, sizeof(int32_t), st)) != cudaSuccess) {
        return e;
    }
    if (n > 0)
        pair_scatter_kernel<<<blocks, 256, 0, st>>>(probes, nq, P, L, skip_len, lstart, lcount,
                                                    lcursor, pair_q, pair_slot);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Merge: per query, the k smallest of its P partial lists by (score, slot, j),
// which is the order (score, probe rank, row in list).  The candidates are first
// cut at tau = the smallest k-th score among full partial lists (every answer is
// <= tau and at least k candidates are), then sorted in shared memory.  If more
// than MCAP survive (massive ties), an exact radix selection over all candidates
// decides instead.
// ---------------------------------------------------------------------------
namespace {
constexpr int MRG_BLOCK = 256;
constexpr int MCAP = 4096;

__device__ void bitonic_u64(unsigned long long* a, int n) {
    for (int k = 2; k <= n; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += MRG_BLOCK) {
                const int p = i ^ j;
                if (p > i) {
                    const unsigned long long x = a[i], y = a[p];
                    if ((x > y) == ((i & k) == 0)) {
                        a[i] = y;
                        a[p] = x;
                    }
                }
            }
            __syncthreads();
        }
}

// rank-th smallest (1-based) 32-bit key among key_of(i), i < n.
template <class F>
__device__ uint32_t radix_select32(F key_of, int64_t n, unsigned rank, unsigned* hist,
                                   unsigned* shv) {
    uint32_t prefix = 0, mask = 0;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = threadIdx.x; i < 256; i += MRG_BLOCK) hist[i] = 0;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < n; i += MRG_BLOCK) {
            const uint32_t k = key_of(i);
            if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned r = rank;
            int b = 0;
            for (; b < 256; ++b) {
                if (r <= hist[b]) break;
                r -= hist[b];
            }
            shv[0] = prefix | ((uint32_t)b << shift);
            shv[1] = r;
        }
        __syncthreads();
        prefix = shv[0];
        rank = shv[1];
        mask |= 255u << shift;
        __syncthreads();
    }
    return prefix;
}

// Candidate i = slot * k + j of query q lives at q * stride_q + slot * stride_slot
// + j.  part_row holds arena rows mapped through row_ids, or, when row_ids is
// null, the ids themselves.
// Exact rescoring (MergeRescore) takes at most this many winners per query.
constexpr int RS_MAX = 128;

// With rescore, the winners leave as arena rows (out_ids) in estimate order for
// rescore_l2_kernel, which writes the final ids and scores.
__global__ void __launch_bounds__(MRG_BLOCK) merge_topk_kernel(
    const float* __restrict__ part_score, const int64_t* __restrict__ part_row,
    const int64_t* __restrict__ row_ids, int P, int k, int64_t stride_q, int64_t stride_slot,
    int64_t rstride_q, int64_t rstride_slot, int64_t* __restrict__ out_ids,
    float* __restrict__ out_scores, int32_t* __restrict__ out_counts, int rescore) {
    __shared__ unsigned long long cand[MCAP];
    __shared__ unsigned hist[256];
    __shared__ unsigned shv[4];
    __shared__ unsigned s_tau, s_cnt, s_valid;
    const int q = blockIdx.x;
    const int64_t n = (int64_t)P * k;
    const float* ps = part_score + (int64_t)q * stride_q;
    const int64_t* pr = part_row + (int64_t)q * rstride_q;
    const float INF = __int_as_float(0x7f800000);
    // candidate i = slot * k + j: its score at ps[at(i)], its row / id at pr[rat(i)]
    auto at = [&](int64_t i) -> int64_t { return (i / k) * stride_slot + (i % k); };
    auto rat = [&](int64_t i) -> int64_t { return (i / k) * rstride_slot + (i % k); };

    // tau: smallest k-th score among full partial lists; count valid candidates
    float tau = INF;
    unsigned nvalid = 0;
    for (int s = threadIdx.x; s < P; s += MRG_BLOCK) {
        const float last = ps[(int64_t)s * stride_slot + k - 1];
        if (score_valid(last)) tau = fminf(tau, last);
    }
    for (int64_t i = threadIdx.x; i < n; i += MRG_BLOCK) nvalid += score_valid(ps[at(i)]) ? 1u : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        tau = fminf(tau, __shfl_xor_sync(0xffffffffu, tau, o));
        nvalid += __shfl_xor_sync(0xffffffffu, nvalid, o);
    }
    if (threadIdx.x == 0) {
        s_tau = float_key(INF);
        s_cnt = 0;
        s_valid = 0;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        atomicMin(&s_tau, float_key(tau));
        atomicAdd(&s_valid, nvalid);
    }
    __syncthreads();
    tau = key_float(s_tau);
    const unsigned total_valid = s_valid;
    const int kk = (int)((unsigned)k < total_valid ? (unsigned)k : total_valid);
    for (int64_t i = threadIdx.x; i < n; i += MRG_BLOCK) {
        const float s = ps[at(i)];
        if (score_valid(s) && s <= tau) {
            const unsigned pos = atomicAdd(&s_cnt, 1u);
            if (pos < (unsigned)MCAP)
                cand[pos] = ((unsigned long long)float_key(s) << 32) | (uint32_t)i;
        }
    }
    __syncthreads();
    const unsigned cnt = s_cnt;
    if (cnt <= (unsigned)MCAP) {
        int n2 = 1;
        while (n2 < (int)cnt) n2 <<= 1;
        for (int i = (int)cnt + threadIdx.x; i < n2; i += MRG_BLOCK) cand[i] = ~0ull;
        __syncthreads();
        bitonic_u64(cand, n2);
    } else {
        // exact selection over all candidates (keys are unique: (score, index))
        auto hi_key = [&](int64_t i) -> uint32_t {
            const float s = ps[at(i)];
            return score_valid(s) ? float_key(s) : 0xffffffffu;
        };
        const uint32_t kh = radix_select32(hi_key, n, (unsigned)kk, hist, shv);
        // m = #candidates with a smaller score key
        if (threadIdx.x == 0) s_cnt = 0;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < n; i += MRG_BLOCK)
            if (hi_key(i) < kh) atomicAdd(&s_cnt, 1u);
        __syncthreads();
        const unsigned m = s_cnt;
        auto lo_key = [&](int64_t i) -> uint32_t {
            return hi_key(i) == kh ? (uint32_t)i : 0xffffffffu;
        };
        const uint32_t kl = radix_select32(lo_key, n, (unsigned)kk - m, hist, shv);
        if (threadIdx.x == 0) s_cnt = 0;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < n; i += MRG_BLOCK) {
            const uint32_t h = hi_key(i);
            if (h < kh || (h == kh && (uint32_t)i <= kl)) {
                const unsigned pos = atomicAdd(&s_cnt, 1u);
                if (pos < (unsigned)MCAP) cand[pos] = ((unsigned long long)h << 32) | (uint32_t)i;
            }
        }
        __syncthreads();
        int n2 = 1;
        while (n2 < kk) n2 <<= 1;
        for (int i = kk + threadIdx.x; i < n2; i += MRG_BLOCK) cand[i] = ~0ull;
        __syncthreads();
        bitonic_u64(cand, n2);
    }
    if (rescore) {
        // hand the winners to rescore_l2_kernel: their arena rows in estimate order
        // (ties: the merge order), the count in out_counts
        for (int j = threadIdx.x; j < k; j += MRG_BLOCK) {
            out_ids[(int64_t)q * k + j] =
                j < kk ? pr[rat((int64_t)(cand[j] & 0xffffffffu))] : (int64_t)-1;
            out_scores[(int64_t)q * k + j] = j < kk ? key_float((uint32_t)(cand[j] >> 32)) : INF;
        }
        if (threadIdx.x == 0) out_counts[q] = kk;
        return;
    }
    for (int j = threadIdx.x; j < k; j += MRG_BLOCK) {
        int64_t id = -1;
        float s = INF;
        if (j < kk) {
            const int64_t i = (int64_t)(cand[j] & 0xffffffffu);
            s = ps[at(i)];
            const int64_t r = pr[rat(i)];
            id = row_ids ? row_ids[r] : r;
        }
        out_ids[(int64_t)q * k + j] = id;
        out_scores[(int64_t)q * k + j] = s;
    }
    if (threadIdx.x == 0) out_counts[q] = kk;
}

// The same merge, one warp per query, for k <= 32 and at most 32 MWL candidates
// per query (the batch shapes of the searches: P k = 320 at P = 32, k = 10):
// the same cut at tau and the same (score, slot, j) order, with the candidates
// in registers and the k winners taken by k rounds of a warp minimum instead of
// a block-wide sort; the winners' ids are then fetched by k lanes at once.
constexpr int MWL = 16;        // candidates per lane
constexpr int MW_WARPS = 8;    // queries per block

__global__ void __launch_bounds__(MW_WARPS * 32) merge_topk_warp_kernel(
    const float* __restrict__ part_score, const int64_t* __restrict__ part_row,
    const int64_t* __restrict__ row_ids, int nq, int P, int k, int64_t stride_q,
    int64_t stride_slot, int64_t rstride_q, int64_t rstride_slot, int64_t* __restrict__ out_ids,
    float* __restrict__ out_scores, int32_t* __restrict__ out_counts) {
    __shared__ uint32_t sel[MW_WARPS][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * MW_WARPS + warp;
    if (q >= nq) return;  // warp-uniform
    const int n = P * k;  // <= 32 MWL (checked by the launcher)
    const float* ps = part_score + (int64_t)q * stride_q;
    const int64_t* pr = part_row + (int64_t)q * rstride_q;
    const float INF = __int_as_float(0x7f800000);
    float tau = INF;
    for (int sl = lane; sl < P; sl += 32) {
        const float last = ps[(int64_t)sl * stride_slot + k - 1];
        if (score_valid(last)) tau = fminf(tau, last);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tau = fminf(tau, __shfl_xor_sync(0xffffffffu, tau, o));
    unsigned long long key[MWL];
    unsigned nvalid = 0;
#pragma unroll
    for (int u = 0; u < MWL; ++u) {
        const int i = lane + 32 * u;
        key[u] = ~0ull;
        if (i < n) {
            const float sv = ps[(int64_t)(i / k) * stride_slot + (i % k)];
            if (score_valid(sv)) {
                ++nvalid;
                if (sv <= tau) key[u] = ((unsigned long long)float_key(sv) << 32) | (uint32_t)i;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) nvalid += __shfl_xor_sync(0xffffffffu, nvalid, o);
    int kk = (int)((unsigned)k < nvalid ? (unsigned)k : nvalid);
    // k rounds: the warp's smallest key leaves its lane (keys are distinct).  At
    // least kk candidates are <= tau (a full list's k entries are); should the
    // lists break that, the answer stops at the candidates there are
    unsigned long long m = ~0ull;
#pragma unroll
    for (int u = 0; u < MWL; ++u) m = key[u] < m ? key[u] : m;
    for (int r = 0; r < kk; ++r) {
        unsigned long long w = m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, w, o);
            w = t < w ? t : w;
        }
        if (w == ~0ull) {  // warp-uniform
            kk = r;
            break;
        }
        if (m == w) {
            sel[warp][r] = (uint32_t)(w & 0xffffffffu);
            m = ~0ull;
#pragma unroll
            for (int u = 0; u < MWL; ++u) {
                if (key[u] == w) key[u] = ~0ull;
                m = key[u] < m ? key[u] : m;
            }
        }
    }
    __syncwarp();
    if (lane < k) {
        int64_t id = -1;
        float sv = INF;
        if (lane < kk) {
            const int i = (int)sel[warp][lane];
            sv = ps[(int64_t)(i / k) * stride_slot + (i % k)];
            const int64_t row = pr[(int64_t)(i / k) * rstride_slot + (i % k)];
            id = row_ids ? row_ids[row] : row;
        }
        out_ids[(int64_t)q * k + lane] = id;
        out_scores[(int64_t)q * k + lane] = sv;
    }
    if (lane == 0) out_counts[q] = kk;
}

bool merge_fits_warp(int P, int k) { return k >= 1 && k <= 32 && (int64_t)P * k <= 32 * MWL; }
}  // namespace

namespace {
// Exact squared L2 of the winners, in the reference's arithmetic: the sum over
// i = 0 .. dim-1 of (q_i - x_i)^2 in index order, each step rounded to fp32
// (Cluster::search_into's distance, AgentMemory/M3/src/cluster.cpp:229-274).
// One block per query, one thread per winner: the thread streams its row from
// HBM in 16-byte loads, 128 bytes per batch with the next batch in flight while
// it sums the current one, against the query staged in shared memory; then the
// winners are sorted by (exact score, estimate rank).
constexpr int RS_QCH = 2048;  // query dims staged per round

__device__ __forceinline__ void unpack16(const uint4& u, float* v, bool bf) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    if (bf) {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            v[2 * h] = __uint_as_float(w[h] << 16);
            v[2 * h + 1] = __uint_as_float(w[h] & 0xffff0000u);
        }
    } else {
#pragma unroll
        for (int h = 0; h < 4; ++h) v[h] = __uint_as_float(w[h]);
    }
}

// Continues e over dims [0, n) of one staged query chunk; src points at the row's
// first dim of the chunk (16-byte aligned), ng16 = 16-byte groups readable there.
template <bool BF>
__device__ __forceinline__ float l2_chunk(const uint4* __restrict__ src, int ng16,
                                          const float* qs, int n, float e) {
    constexpr int EPG = BF ? 8 : 4;  // elements per 16-byte group
    constexpr int U = 8;             // groups per batch (128 bytes)
    const int G = (n + EPG - 1) / EPG;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    uint4 cur[U], nxt[U];
#pragma unroll
    for (int u = 0; u < U; ++u) cur[u] = u < G && u < ng16 ? __ldg(src + u) : z;
    for (int g0 = 0; g0 < G; g0 += U) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int g = g0 + U + u;
            nxt[u] = g < G && g < ng16 ? __ldg(src + g) : z;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float v[8], qv[8];
            unpack16(cur[u], v, BF);
            // the group's query values by 16-byte broadcast reads (every lane reads
            // the same address); values past n are read but never summed
            const float4* q4 = reinterpret_cast<const float4*>(qs + (g0 + u) * EPG);
#pragma unroll
            for (int h4 = 0; h4 < EPG / 4; ++h4) {
                const float4 a = q4[h4];
                qv[4 * h4] = a.x;
                qv[4 * h4 + 1] = a.y;
                qv[4 * h4 + 2] = a.z;
                qv[4 * h4 + 3] = a.w;
            }
#pragma unroll
            for (int h = 0; h < EPG; ++h) {
                const int i = (g0 + u) * EPG + h;
                if (i < n) {
                    const float df = __fsub_rn(qv[h], v[h]);
                    e = __fadd_rn(e, __fmul_rn(df, df));
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) cur[u] = nxt[u];
    }
    return e;
}

template <bool BF>
__global__ void __launch_bounds__(RS_MAX) rescore_l2_kernel(MergeRescore rs,
                                                           const int64_t* __restrict__ row_ids,
                                                           int k, int64_t* __restrict__ out_ids,
                                                           float* __restrict__ out_scores,
                                                           const int32_t* __restrict__ out_counts) {
    __shared__ __align__(16) float qs[RS_QCH];
    __shared__ unsigned long long key[RS_MAX];
    __shared__ int64_t wrow[RS_MAX];
    const int q = blockIdx.x, j = threadIdx.x;
    const int kk = min(out_counts[q], k);
    const int64_t row = j < kk ? out_ids[(int64_t)q * k + j] : -1;
    wrow[j] = row;
    const float* qr = rs.Q + (int64_t)q * rs.ldq;
    const size_t esz = BF ? 2 : 4;
    const unsigned char* base = static_cast<const unsigned char*>(rs.rows);
    float e = 0.f;
    for (int d0 = 0; d0 < rs.dim; d0 += RS_QCH) {
        const int n = min(RS_QCH, rs.dim - d0);
        __syncthreads();
        for (int i = j; i < n; i += RS_MAX) qs[i] = qr[d0 + i];
        __syncthreads();
        if (row >= 0) {
            const uint4* src = reinterpret_cast<const uint4*>(base + ((size_t)row * rs.row_ld + d0) * esz);
            const int ng16 = (int)(((rs.row_ld - d0) * (int64_t)esz) / 16);
            e = l2_chunk<BF>(src, ng16, qs, n, e);
        }
    }
    key[j] = j < kk ? (((unsigned long long)float_key(e) << 32) | (uint32_t)j) : ~0ull;
    __syncthreads();
    // bitonic sort of the RS_MAX keys, one per thread
    for (int s2 = 2; s2 <= RS_MAX; s2 <<= 1)
        for (int h = s2 >> 1; h > 0; h >>= 1) {
            const int p = j ^ h;
            unsigned long long a = key[j], b = key[p];
            __syncthreads();
            if (p > j) {
                if ((a > b) == ((j & s2) == 0)) {
                    key[j] = b;
                    key[p] = a;
                }
            }
            __syncthreads();
        }
    if (j < k) {
        int64_t id = -1;
        float sc = __int_as_float(0x7f800000);
        if (j < kk) {
            const unsigned long long c = key[j];
            sc = key_float((uint32_t)(c >> 32));
            id = row_ids[wrow[(uint32_t)(c & 0xffffffffu)]];
        }
        out_ids[(int64_t)q * k + j] = id;
        out_scores[(int64_t)q * k + j] = sc;
    }
}
}  // namespace

cudaError_t launch_merge_topk(const float* part_score, const int64_t* part_row,
                              const int64_t* row_ids, int nq, int P, int k, int64_t* out_ids,
                              float* out_scores, int32_t* out_counts, cudaStream_t st,
                              const MergeRescore* rs) {
    if (nq <= 0) return cudaSuccess;
    if (rs && (k > RS_MAX || !row_ids)) return cudaErrorInvalidValue;
    if (!rs && merge_fits_warp(P, k)) {
        merge_topk_warp_kernel<<<(nq + MW_WARPS - 1) / MW_WARPS, MW_WARPS * 32, 0, st>>>(
            part_score, part_row, row_ids, nq, P, k, (int64_t)P * k, k, (int64_t)P * k, k,
            out_ids, out_scores, out_counts);
        return cudaGetLastError();
    }
    merge_topk_kernel<<<nq, MRG_BLOCK, 0, st>>>(part_score, part_row, row_ids, P, k,
                                                (int64_t)P * k, k, (int64_t)P * k, k, out_ids,
                                                out_scores, out_counts, rs ? 1 : 0);
    if (rs) {
        if (rs->bf16_rows)
            rescore_l2_kernel<true><<<nq, RS_MAX, 0, st>>>(*rs, row_ids, k, out_ids, out_scores,
                                                           out_counts);
        else
            rescore_l2_kernel<false><<<nq, RS_MAX, 0, st>>>(*rs, row_ids, k, out_ids, out_scores,
                                                            out_counts);
    }
    return cudaGetLastError();
}

namespace {
__global__ void clear_partials_kernel(float* __restrict__ s, int64_t* __restrict__ r, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        s[i] = __int_as_float(0x7f800000);
        r[i] = -1;
    }
}
}  // namespace

cudaError_t launch_clear_partials(float* part_score, int64_t* part_row, int64_t n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 4096);
    clear_partials_kernel<<<(unsigned)blocks, 256, 0, st>>>(part_score, part_row, n);
    return cudaGetLastError();
}

cudaError_t launch_merge_shards(const float* scores, const int64_t* ids, int nshard, int nq, int k,
                                int64_t* out_ids, float* out_scores, int32_t* out_counts,
                                cudaStream_t st) {
    if (nq <= 0 || k <= 0) return cudaSuccess;
    if (merge_fits_warp(nshard, k)) {
        merge_topk_warp_kernel<<<(nq + MW_WARPS - 1) / MW_WARPS, MW_WARPS * 32, 0, st>>>(
            scores, ids, nullptr, nq, nshard, k, k, (int64_t)nq * k, k, (int64_t)nq * k, out_ids,
            out_scores, out_counts);
        return cudaGetLastError();
    }
    merge_topk_kernel<<<nq, MRG_BLOCK, 0, st>>>(scores, ids, nullptr, nshard, k, k,
                                                (int64_t)nq * k, k, (int64_t)nq * k, out_ids,
                                                out_scores, out_counts, 0);
    return cudaGetLastError();
}

cudaError_t launch_merge_shards_packed(const unsigned char* packed, int nshard, int nq, int k,
                                       int64_t shard_bytes, int64_t ids_offset, int64_t* out_ids,
                                       float* out_scores, int32_t* out_counts, cudaStream_t st) {
    if (nq <= 0 || k <= 0) return cudaSuccess;
    if (shard_bytes % 8 || ids_offset % 8 || (reinterpret_cast<uintptr_t>(packed) & 7) ||
        ids_offset < (int64_t)nq * k * 4 || shard_bytes < ids_offset + (int64_t)nq * k * 8)
        return cudaErrorInvalidValue;
    const float* sc = reinterpret_cast<const float*>(packed);
    const int64_t* ids = reinterpret_cast<const int64_t*>(packed + ids_offset);
    if (merge_fits_warp(nshard, k)) {
        merge_topk_warp_kernel<<<(nq + MW_WARPS - 1) / MW_WARPS, MW_WARPS * 32, 0, st>>>(
            sc, ids, nullptr, nq, nshard, k, k, shard_bytes / 4, k, shard_bytes / 8, out_ids,
            out_scores, out_counts);
        return cudaGetLastError();
    }
    merge_topk_kernel<<<nq, MRG_BLOCK, 0, st>>>(sc, ids, nullptr, nshard, k, k, shard_bytes / 4, k,
                                                shard_bytes / 8, out_ids, out_scores, out_counts, 0);
    return cudaGetLastError();
}

}  // namespace m3g
