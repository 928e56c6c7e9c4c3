// engine.cu -- host implementation of the m3gpu engine (see engine.h).
//
// Reference behaviour mirrored here, by file:
//   AgentMemory/M3/src/cluster.cpp   add/update/erase/rebuild/compact of one list
//   AgentMemory/M3/src/m3_index.cpp  set_centroids, add_cluster, set_centroid,
//                                    nearest_clusters, search_on, search_nprobe,
//                                    maintenance_pass
//   AgentMemory/M3/src/m3_async.cpp  create_ivf, start/stop, queue + writers,
//                                    flush, search, load_cluster,
//                                    enqueue_insert_auto, *_of
#include "engine.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <chrono>
#include <cmath>
#include <cstring>
#include <numeric>
#include <unordered_set>

#include "kernels_kmeans.h"

namespace m3g {

[[noreturn]] void fail(int code, const std::string& msg) { throw Error(code, msg); }

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(M3G_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
    }
}

// Never throws (it also runs in destructors); a failed switch surfaces at the
// next CUDA call, which does check.
DeviceGuard::DeviceGuard(int dev) {
    if (cudaGetDevice(&prev_) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    if (prev_ != dev) {
        if (cudaSetDevice(dev) == cudaSuccess) changed_ = true;
        else cudaGetLastError();
    }
}
DeviceGuard::~DeviceGuard() {
    if (changed_) cudaSetDevice(prev_);
}

void sample_rows(uint64_t seed, int64_t n, int64_t m, int64_t* out) {
    if (m < 0 || m > n) fail(M3G_EINVAL, "sample_rows: need 0 <= m <= n");
    std::vector<int64_t> perm((size_t)n);
    std::iota(perm.begin(), perm.end(), int64_t(0));
    uint64_t st = seed;
    auto next = [&st]() {
        uint64_t z = (st += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    for (int64_t i = 0; i < m; ++i) {
        const int64_t j = i + (int64_t)(next() % (uint64_t)(n - i));
        std::swap(perm[(size_t)i], perm[(size_t)j]);
        out[i] = perm[(size_t)i];
    }
}

namespace {

constexpr int kDefaultNsm = 148;

int round_up4(int d) { return (d + 3) & ~3; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

}  // namespace

void encode_tma_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                   uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                   CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) fail(M3G_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t gdim[2] = {(cuuint64_t)inner, (cuuint64_t)std::max<uint64_t>(rows, 1)};
    cuuint64_t gstride[1] = {(cuuint64_t)row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void*>(base), gdim, gstride, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        fail(M3G_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

namespace {

// 2-D tensor map over the arena's [rows, ldr] elements, boxes of 128 bytes
// (32 fp32 or 64 bf16) x h rows, 128-byte swizzle.
void make_row_map(CUtensorMap* m, const Index& ix, int h) {
    if (ix.bf16_rows())
        encode_tma_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, ix.vecs.p, (uint64_t)ix.ldr,
                      (uint64_t)ix.arena_cap, (uint64_t)ix.ldr * 2, 64, (uint32_t)h,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    else
        encode_tma_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ix.vecs.p, (uint64_t)ix.ldr,
                      (uint64_t)ix.arena_cap, (uint64_t)ix.ldr * 4, 32, (uint32_t)h,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

// Which kernel scans the lists: the tensor-core scan (default, where it
// applies) or the SIMT scan (M3G_SCAN=simt).  Both rank by (score, probe slot,
// row); their scores differ only in fp32 rounding.
bool use_tc_scan() {
    static const bool tc = [] {
        const char* v = std::getenv("M3G_SCAN");
        return !(v && std::string(v) == "simt");
    }();
    return tc;
}

// Which GEMM produces the approximate coarse scores: the tcgen05 bf16x3 kernel
// (default) or the SIMT fp32 kernel (M3G_COARSE_GEMM=simt).  Either way the
// selection is exact; only its error bound (and so the candidate count) differs.
bool use_tc_gemm() {
    static const bool tc = [] {
        const char* v = std::getenv("M3G_COARSE_GEMM");
        return !(v && std::string(v) == "simt");
    }();
    return tc;
}

// S[M, N] ~ A . B^T for fp32 rows A [M, lda], B [N, ldb] (dpad wide).  On the
// tensor-core path A3 / B3 are the split operands ([M|N, kp] bf16) the caller
// prepared.  Returns the bound factor beta of the approximation.
float coarse_gemm(const float* A, int64_t lda, const __nv_bfloat16* A3, const float* B,
                  int64_t ldb, const __nv_bfloat16* B3, float* S, int64_t lds, int M, int N,
                  int dpad, int* err, cudaStream_t st) {
    // a few rows: a GEMV over every SM beats the tiled GEMMs (which give one row
    // tile a few CTAs), with the SIMT GEMM's error bound
    if (gemv_fits(A, lda, B, ldb, M, dpad)) {
        int dev = 0, sms = 148;
        M3G_CK(cudaGetDevice(&dev));
        M3G_CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        launch_gemv_nt(A, lda, B, ldb, S, lds, M, N, dpad, sms, st);
        M3G_CK(cudaGetLastError());
        return sgemm_error_beta(dpad);
    }
    if (use_tc_gemm()) {
        const int kp = gemm_tc_kdim(dpad);
        CUtensorMap ma, mb;
        encode_tma_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, A3, (uint64_t)kp, (uint64_t)M,
                      (uint64_t)kp * 2, (uint32_t)gemm_tc_box_k(), (uint32_t)gemm_tc_box_rows_a(),
                      CU_TENSOR_MAP_SWIZZLE_128B);
        encode_tma_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, B3, (uint64_t)kp, (uint64_t)N,
                      (uint64_t)kp * 2, (uint32_t)gemm_tc_box_k(), (uint32_t)gemm_tc_box_rows_b(),
                      CU_TENSOR_MAP_SWIZZLE_128B);
        M3G_CK(launch_gemm_tc(ma, mb, S, lds, M, N, kp, err, st));
        return gemm_tc_error_beta(dpad);
    }
    launch_sgemm_nt(A, lda, B, ldb, S, lds, M, N, dpad, st);
    M3G_CK(cudaGetLastError());
    return sgemm_error_beta(dpad);
}

void rebuild_maps(Index& ix) {
    if (!ix.vecs.p) {
        ix.maps_valid = false;
        return;
    }
    make_row_map(&ix.maps.m128, ix, 128);
    make_row_map(&ix.maps.m64, ix, 64);
    make_row_map(&ix.maps.m32, ix, 32);
    make_row_map(&ix.maps.m16, ix, 16);
    make_row_map(&ix.maps.m8, ix, 8);
    ix.maps_valid = true;
}

// Copies n host rows of `dim` floats into device rows of `dpad` floats.
void h2d_rows(float* dst, int dpad, const float* src, int dim, int64_t n, cudaStream_t st) {
    if (n <= 0) return;
    M3G_CK(cudaMemcpy2DAsync(dst, (size_t)dpad * 4, src, (size_t)dim * 4, (size_t)dim * 4,
                             (size_t)n, cudaMemcpyHostToDevice, st));
}

// ---------------- index device state ----------------

void ensure_centroid_cap(Index& ix, size_t need) {
    if (need <= ix.c_cap && ix.C.p) return;
    size_t cap = std::max<size_t>({need, ix.c_cap * 2, 16});
    DBuf<float> C, cn, cn2;
    DBuf<__nv_bfloat16> C3;
    DBuf<int64_t> off;
    DBuf<int32_t> len, order;
    const int kp = gemm_tc_kdim(ix.dpad);
    C.alloc(cap * ix.dpad);
    C3.alloc(cap * (size_t)kp);
    cn.alloc(cap);
    cn2.alloc(cap);
    off.alloc(cap);
    len.alloc(cap);
    order.alloc(cap);
    M3G_CK(cudaMemsetAsync(C.p, 0, cap * ix.dpad * 4, ix.wstream));
    if (ix.C.p && ix.c_cap) {
        M3G_CK(cudaMemcpyAsync(C.p, ix.C.p, ix.c_cap * ix.dpad * 4, cudaMemcpyDeviceToDevice, ix.wstream));
        M3G_CK(cudaMemcpyAsync(cn.p, ix.cn.p, ix.c_cap * 4, cudaMemcpyDeviceToDevice, ix.wstream));
        M3G_CK(cudaMemcpyAsync(cn2.p, ix.cn2.p, ix.c_cap * 4, cudaMemcpyDeviceToDevice, ix.wstream));
        M3G_CK(cudaMemcpyAsync(C3.p, ix.C3.p, ix.c_cap * (size_t)kp * 2, cudaMemcpyDeviceToDevice,
                               ix.wstream));
    }
    M3G_CK(cudaStreamSynchronize(ix.wstream));
    ix.C.swap(C);
    ix.C3.swap(C3);
    ix.cn.swap(cn);
    ix.cn2.swap(cn2);
    ix.d_list_off.swap(off);
    ix.d_list_len.swap(len);
    ix.d_list_order.swap(order);
    ix.c_cap = cap;
}

// Uploads centroids [c0, c0+n) from the host copy and recomputes their norms.
void upload_centroids(Index& ix, int c0, int n) {
    if (n <= 0) return;
    h2d_rows(ix.C.p + (size_t)c0 * ix.dpad, ix.dpad, ix.centroids.data() + (size_t)c0 * ix.dim,
             ix.dim, n, ix.wstream);
    launch_row_norms(ix.C.p + (size_t)c0 * ix.dpad, ix.dpad, n, ix.dim, ix.cn.p + c0, ix.cn2.p + c0,
                     ix.wstream);
    M3G_CK(cudaGetLastError());
    const int kp = gemm_tc_kdim(ix.dpad);
    M3G_CK(launch_split3(ix.C.p + (size_t)c0 * ix.dpad, ix.dpad, n, ix.dpad, kp,
                         ix.C3.p + (size_t)c0 * kp, true, ix.wstream));
}

// Uploads per-list offsets / lengths and the longest-first order.
void refresh_list_meta(Index& ix) {
    const int L = ix.nlist();
    if (L == 0) return;
    std::vector<int64_t> off(L);
    std::vector<int32_t> len(L), order(L);
    for (int l = 0; l < L; ++l) {
        off[l] = ix.lists[l].off;
        len[l] = (int32_t)ix.lists[l].len;
    }
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return len[a] > len[b]; });
    M3G_CK(cudaMemcpyAsync(ix.d_list_off.p, off.data(), L * 8, cudaMemcpyHostToDevice, ix.wstream));
    M3G_CK(cudaMemcpyAsync(ix.d_list_len.p, len.data(), L * 4, cudaMemcpyHostToDevice, ix.wstream));
    M3G_CK(cudaMemcpyAsync(ix.d_list_order.p, order.data(), L * 4, cudaMemcpyHostToDevice, ix.wstream));
    M3G_CK(cudaStreamSynchronize(ix.wstream));
}

// Reallocates the arena with room for `extra` more rows, laying every list out
// again contiguously (this also reclaims the holes relocations leave behind).
void grow_arena(Index& ix, int64_t extra) {
    int64_t used = 0;
    for (auto& l : ix.lists) used += l.cap;
    const int64_t cap = std::max<int64_t>({used + extra, ix.arena_cap + ix.arena_cap / 2, 1024});
    DBuf<float> vecs, rn;
    DBuf<int64_t> ids;
    DBuf<uint8_t> alive;
    const int64_t rb = ix.row_bytes();
    vecs.alloc((size_t)(cap * rb / 4));
    rn.alloc((size_t)cap);
    ids.alloc((size_t)cap);
    alive.alloc((size_t)cap);
    M3G_CK(cudaMemsetAsync(vecs.p, 0, (size_t)(cap * rb), ix.wstream));
    M3G_CK(cudaMemsetAsync(alive.p, 0, (size_t)cap, ix.wstream));
    int64_t pos = 0;
    for (auto& l : ix.lists) {
        if (l.len > 0) {
            M3G_CK(cudaMemcpyAsync(reinterpret_cast<unsigned char*>(vecs.p) + pos * rb,
                                   ix.row_ptr(l.off), (size_t)(l.len * rb),
                                   cudaMemcpyDeviceToDevice, ix.wstream));
            M3G_CK(cudaMemcpyAsync(rn.p + pos, ix.rnorm2.p + l.off, (size_t)l.len * 4,
                                   cudaMemcpyDeviceToDevice, ix.wstream));
            M3G_CK(cudaMemcpyAsync(ids.p + pos, ix.ids.p + l.off, (size_t)l.len * 8,
                                   cudaMemcpyDeviceToDevice, ix.wstream));
            M3G_CK(cudaMemcpyAsync(alive.p + pos, ix.alive.p + l.off, (size_t)l.len,
                                   cudaMemcpyDeviceToDevice, ix.wstream));
        }
        l.off = pos;
        pos += l.cap;
    }
    M3G_CK(cudaStreamSynchronize(ix.wstream));
    ix.vecs.swap(vecs);
    ix.rnorm2.swap(rn);
    ix.ids.swap(ids);
    ix.alive.swap(alive);
    ix.arena_cap = cap;
    ix.arena_used = pos;
    rebuild_maps(ix);
}

// Gives list l a fresh segment of `cap` rows, keeping its first `keep` rows.
// When the arena is full it is rebuilt with every list laid out again, this
// one already at its new capacity.
void relocate(Index& ix, int l, int64_t cap, int64_t keep) {
    ListMeta& L = ix.lists[l];
    if (ix.arena_used + cap > ix.arena_cap) {
        L.cap = cap;
        grow_arena(ix, 0);
        return;
    }
    const int64_t dst = ix.arena_used;
    if (keep > 0) {
        M3G_CK(cudaMemcpyAsync(ix.row_ptr(dst), ix.row_ptr(L.off), (size_t)(keep * ix.row_bytes()),
                               cudaMemcpyDeviceToDevice, ix.wstream));
        M3G_CK(cudaMemcpyAsync(ix.rnorm2.p + dst, ix.rnorm2.p + L.off, (size_t)keep * 4,
                               cudaMemcpyDeviceToDevice, ix.wstream));
        M3G_CK(cudaMemcpyAsync(ix.ids.p + dst, ix.ids.p + L.off, (size_t)keep * 8,
                               cudaMemcpyDeviceToDevice, ix.wstream));
        M3G_CK(cudaMemcpyAsync(ix.alive.p + dst, ix.alive.p + L.off, (size_t)keep,
                               cudaMemcpyDeviceToDevice, ix.wstream));
    }
    L.off = dst;
    L.cap = cap;
    ix.arena_used += cap;
}

void ensure_list_room(Index& ix, int l, int64_t need_len) {
    ListMeta& L = ix.lists[l];
    if (need_len <= L.cap) return;
    const int64_t cap = std::max<int64_t>({need_len, L.cap * 2, 16});
    relocate(ix, l, cap, L.len);
}

// Device rows stage [n, dpad] fp32 (zero padded; a bf16 index rounds them in
// place) into the arena format at device rows dst, with their squared norms (of
// the stored values) into nrm2[n].
void store_staged_rows(Index& ix, unsigned char* dst, float* stage, int64_t n, float* nrm2) {
    if (n <= 0) return;
    if (ix.bf16_rows()) M3G_CK(launch_round_bf16_rows(stage, ix.dpad, n, ix.dim, ix.wstream));
    launch_row_norms(stage, ix.dpad, n, ix.dim, nullptr, nrm2, ix.wstream);
    M3G_CK(cudaGetLastError());
    if (ix.bf16_rows())
        M3G_CK(launch_pack_bf16_rows(stage, ix.dpad, n, ix.dim,
                                     reinterpret_cast<__nv_bfloat16*>(dst), ix.ldr, ix.wstream));
    else
        M3G_CK(cudaMemcpyAsync(dst, stage, (size_t)(n * ix.dpad) * 4, cudaMemcpyDeviceToDevice,
                               ix.wstream));
}

// Host rows [n, dim] fp32 into the arena format at device rows dst (fp32 rows
// copied straight in; bf16 rows staged as fp32, rounded, packed), with their
// squared norms into nrm2[n].
void store_rows(Index& ix, unsigned char* dst, const float* vecs, int64_t n, float* nrm2) {
    if (n <= 0) return;
    if (!ix.bf16_rows()) {
        float* d = reinterpret_cast<float*>(dst);
        h2d_rows(d, ix.ldr, vecs, ix.dim, n, ix.wstream);
        launch_row_norms(d, ix.ldr, n, ix.dim, nullptr, nrm2, ix.wstream);
        M3G_CK(cudaGetLastError());
        return;
    }
    DBuf<float> stage;
    stage.alloc((size_t)(n * ix.dpad));
    if (ix.dpad != ix.dim) M3G_CK(cudaMemsetAsync(stage.p, 0, (size_t)(n * ix.dpad) * 4, ix.wstream));
    h2d_rows(stage.p, ix.dpad, vecs, ix.dim, n, ix.wstream);
    store_staged_rows(ix, dst, stage.p, n, nrm2);
    M3G_CK(cudaStreamSynchronize(ix.wstream));  // the staging buffer is freed on return
}

// Writes rows (ids, host vectors) at arena rows [row0, row0 + n) of list l.
void write_rows(Index& ix, int64_t row0, const int64_t* ids, const float* vecs, int64_t n) {
    if (n <= 0) return;
    M3G_CK(cudaMemcpyAsync(ix.ids.p + row0, ids, (size_t)n * 8, cudaMemcpyHostToDevice, ix.wstream));
    M3G_CK(cudaMemsetAsync(ix.alive.p + row0, 1, (size_t)n, ix.wstream));
    store_rows(ix, ix.row_ptr(row0), vecs, n, ix.rnorm2.p + row0);
}

// Host-side staging of int64 index arrays for the scatter / gather kernels.
struct DevIdx {
    DBuf<int64_t> d;
    void upload(const std::vector<int64_t>& v, cudaStream_t st) {
        d.alloc(v.size());
        if (!v.empty())
            M3G_CK(cudaMemcpyAsync(d.p, v.data(), v.size() * 8, cudaMemcpyHostToDevice, st));
    }
};

// Cluster::rebuild_from (cluster.cpp:152-178): full replace; later duplicates
// of an id keep the first row in the map (unordered_map::emplace).
void list_rebuild(Index& ix, int l, const int64_t* ids, const float* vecs, int64_t n) {
    ListMeta& L = ix.lists[l];
    if (n > L.cap) relocate(ix, l, std::max<int64_t>(n, 16), 0);
    write_rows(ix, L.off, ids, vecs, n);
    L.len = n;
    L.live = n;
    L.ids.assign(ids, ids + n);
    L.alive.assign((size_t)n, 1);
    L.id2row.clear();
    L.id2row.reserve((size_t)n);
    for (int64_t r = 0; r < n; ++r) L.id2row.emplace(ids[r], r);
}

// Cluster::rebuild_from with the rows on the device: d_vecs [n, dim] fp32 or
// bf16 bits (dtype), d_ids [n].  The ids come to the host for the id map.
void list_rebuild_device(Index& ix, int l, const int64_t* d_ids, const void* d_vecs, int dtype,
                         int64_t n) {
    std::vector<int64_t> ids((size_t)n);
    if (n > 0)
        M3G_CK(cudaMemcpyAsync(ids.data(), d_ids, (size_t)n * 8, cudaMemcpyDeviceToHost, ix.wstream));
    ListMeta& L = ix.lists[l];
    if (n > L.cap) relocate(ix, l, std::max<int64_t>(n, 16), 0);
    if (n > 0) {
        DBuf<float> stage;
        stage.alloc((size_t)(n * ix.dpad));
        if (dtype == M3G_BF16) {
            M3G_CK(launch_unpack_bf16_rows(static_cast<const __nv_bfloat16*>(d_vecs), ix.dim, n,
                                           ix.dim, stage.p, ix.dpad, ix.wstream));
        } else {
            if (ix.dpad != ix.dim)
                M3G_CK(cudaMemsetAsync(stage.p, 0, (size_t)(n * ix.dpad) * 4, ix.wstream));
            M3G_CK(cudaMemcpy2DAsync(stage.p, (size_t)ix.dpad * 4, d_vecs, (size_t)ix.dim * 4,
                                     (size_t)ix.dim * 4, (size_t)n, cudaMemcpyDeviceToDevice,
                                     ix.wstream));
        }
        store_staged_rows(ix, ix.row_ptr(L.off), stage.p, n, ix.rnorm2.p + L.off);
        M3G_CK(cudaMemcpyAsync(ix.ids.p + L.off, d_ids, (size_t)n * 8, cudaMemcpyDeviceToDevice,
                               ix.wstream));
        M3G_CK(cudaMemsetAsync(ix.alive.p + L.off, 1, (size_t)n, ix.wstream));
        M3G_CK(cudaStreamSynchronize(ix.wstream));
    }
    L.len = n;
    L.live = n;
    L.ids = std::move(ids);
    L.alive.assign((size_t)n, 1);
    L.id2row.clear();
    L.id2row.reserve((size_t)n);
    for (int64_t r = 0; r < n; ++r) L.id2row.emplace(L.ids[(size_t)r], r);
}

// Cluster::add_batch (cluster.cpp:55-101).
void list_add(Index& ix, int l, const int64_t* ids, const float* vecs, int64_t n) {
    if (!ids || !vecs || n == 0) return;
    ListMeta& L = ix.lists[l];
    {
        std::unordered_set<int64_t> seen;
        seen.reserve((size_t)n * 2);
        for (int64_t r = 0; r < n; ++r) {
            if (!seen.insert(ids[r]).second)
                fail(M3G_ERUNTIME, "Cluster::add_batch: duplicate id in batch");
            if (L.id2row.count(ids[r])) fail(M3G_ERUNTIME, "Cluster::add_batch: duplicate id exists");
        }
    }
    ensure_list_room(ix, l, L.len + n);
    write_rows(ix, L.off + L.len, ids, vecs, n);
    for (int64_t r = 0; r < n; ++r) {
        L.id2row.emplace(ids[r], L.len + r);
        L.ids.push_back(ids[r]);
        L.alive.push_back(1);
    }
    L.len += n;
    L.live += n;
}

// Cluster::add_batch for many lists at once (the per-cluster ops of
// enqueue_insert_auto, m3_async.cpp:262-313): rows grouped by list (ascending
// list id, call order within a list); a list whose rows repeat an id, in the
// batch or in the list, is skipped and reported through on_error, as its own
// add_batch would have thrown.  Lists that outgrow their segment move first (at
// most one arena rebuild), then every row is staged once and scattered to its
// arena row with its id, tombstone and norm.
template <class OnError>
void list_add_routed(Index& ix, const std::vector<int64_t>& ids, const std::vector<float>& vecs,
                     const std::vector<int32_t>& clusters, OnError on_error) {
    const int64_t n = (int64_t)ids.size();
    if (n == 0) return;
    const int L = ix.nlist();
    std::vector<int64_t> cnt((size_t)L + 1, 0);
    for (int64_t i = 0; i < n; ++i) {
        const int c = clusters[(size_t)i];
        if (c < 0 || c >= L) {
            on_error("IVFIndex::add_batch: invalid cluster_id");
            return;
        }
        cnt[(size_t)c + 1]++;
    }
    for (int l = 0; l < L; ++l) cnt[(size_t)l + 1] += cnt[(size_t)l];
    std::vector<int64_t> order((size_t)n);
    {
        std::vector<int64_t> cur(cnt.begin(), cnt.end() - 1);
        for (int64_t i = 0; i < n; ++i) order[(size_t)cur[(size_t)clusters[(size_t)i]]++] = i;
    }
    // duplicate checks per list (Cluster::add_batch, cluster.cpp:55-101)
    std::vector<char> ok((size_t)L, 1);
    std::vector<int> touched;
    for (int l = 0; l < L; ++l) {
        const int64_t b = cnt[(size_t)l], e = cnt[(size_t)l + 1];
        if (b == e) continue;
        ListMeta& M = ix.lists[(size_t)l];
        std::unordered_set<int64_t> seen;
        seen.reserve((size_t)(e - b) * 2);
        for (int64_t j = b; j < e && ok[(size_t)l]; ++j) {
            const int64_t id = ids[(size_t)order[(size_t)j]];
            if (!seen.insert(id).second) {
                on_error("Cluster::add_batch: duplicate id in batch");
                ok[(size_t)l] = 0;
            } else if (M.id2row.count(id)) {
                on_error("Cluster::add_batch: duplicate id exists");
                ok[(size_t)l] = 0;
            }
        }
        if (ok[(size_t)l]) touched.push_back(l);
    }
    // room: lists that outgrow their segment get max(need, 2 cap, 16) rows
    int64_t extra = 0;
    std::vector<std::pair<int, int64_t>> moves;
    for (int l : touched) {
        ListMeta& M = ix.lists[(size_t)l];
        const int64_t need = M.len + cnt[(size_t)l + 1] - cnt[(size_t)l];
        if (need > M.cap) {
            const int64_t cap = std::max<int64_t>({need, M.cap * 2, 16});
            moves.emplace_back(l, cap);
            extra += cap;
        }
    }
    if (!moves.empty()) {
        if (ix.arena_used + extra > ix.arena_cap) {
            // one rebuild lays every list out again, these at their new capacity
            for (auto& mv : moves) ix.lists[(size_t)mv.first].cap = mv.second;
            grow_arena(ix, 0);
        } else {
            // every moved list to a fresh segment at the arena's end, in one kernel
            std::vector<int64_t> src, dstr;
            for (auto& mv : moves) {
                ListMeta& M = ix.lists[(size_t)mv.first];
                const int64_t to = ix.arena_used;
                for (int64_t r = 0; r < M.len; ++r) {
                    src.push_back(M.off + r);
                    dstr.push_back(to + r);
                }
                M.off = to;
                M.cap = mv.second;
                ix.arena_used += mv.second;
            }
            if (!src.empty()) {
                DevIdx ds, dd;
                ds.upload(src, ix.wstream);
                dd.upload(dstr, ix.wstream);
                M3G_CK(launch_move_rows(ix.vecs.p, ix.row_words(), ix.rnorm2.p, ix.ids.p,
                                        ix.alive.p, ds.d.p, dd.d.p, (int64_t)src.size(),
                                        ix.wstream));
                M3G_CK(cudaStreamSynchronize(ix.wstream));
            }
        }
    }
    // destination arena rows of the kept rows, in staging order
    std::vector<int64_t> dst, src_rows;
    dst.reserve((size_t)n);
    src_rows.reserve((size_t)n);
    for (int l : touched) {
        ListMeta& M = ix.lists[(size_t)l];
        const int64_t b = cnt[(size_t)l], e = cnt[(size_t)l + 1];
        for (int64_t j = b; j < e; ++j) {
            const int64_t i = order[(size_t)j];
            const int64_t row = M.len + (j - b);
            dst.push_back(M.off + row);
            src_rows.push_back(i);
            M.id2row.emplace(ids[(size_t)i], row);
            M.ids.push_back(ids[(size_t)i]);
            M.alive.push_back(1);
        }
        M.len += e - b;
        M.live += e - b;
    }
    const int64_t m = (int64_t)dst.size();
    if (m == 0) return;
    std::vector<float> staging((size_t)(m * ix.dim));
    std::vector<int64_t> row_ids((size_t)m);
    for (int64_t j = 0; j < m; ++j) {
        std::memcpy(&staging[(size_t)(j * ix.dim)], &vecs[(size_t)(src_rows[(size_t)j] * ix.dim)],
                    sizeof(float) * ix.dim);
        row_ids[(size_t)j] = ids[(size_t)src_rows[(size_t)j]];
    }
    DBuf<float> d_src, nrm;
    d_src.alloc((size_t)(m * ix.row_bytes() / 4));
    nrm.alloc((size_t)m);
    if (ix.ldr != ix.dim || ix.bf16_rows())
        M3G_CK(cudaMemsetAsync(d_src.p, 0, (size_t)(m * ix.row_bytes()), ix.wstream));
    store_rows(ix, reinterpret_cast<unsigned char*>(d_src.p), staging.data(), m, nrm.p);
    DevIdx di, dids;
    di.upload(dst, ix.wstream);
    dids.upload(row_ids, ix.wstream);
    const int w = ix.row_words();
    M3G_CK(launch_scatter_rows(d_src.p, w, di.d.p, m, w, ix.vecs.p, w, ix.wstream));
    M3G_CK(launch_scatter_i64(dids.d.p, di.d.p, m, ix.ids.p, ix.wstream));
    M3G_CK(launch_set_bytes(ix.alive.p, di.d.p, m, 1, ix.wstream));
    M3G_CK(launch_scatter_rows(nrm.p, 1, di.d.p, m, 1, ix.rnorm2.p, 1, ix.wstream));
    M3G_CK(cudaStreamSynchronize(ix.wstream));
}

// Cluster::update_batch (cluster.cpp:103-133): rows apply in order; a missing
// id without insert_if_absent raises after the earlier rows were applied.
void list_update(Index& ix, int l, const int64_t* ids, const float* vecs, int64_t n,
                 bool insert_if_absent) {
    if (!ids || !vecs || n == 0) return;
    ListMeta& L = ix.lists[l];
    std::unordered_map<int64_t, int64_t> dst_src;  // list row -> last source row
    std::vector<int64_t> appended;                  // source rows appended, in order
    bool missing = false;
    int64_t r = 0;
    for (; r < n; ++r) {
        auto it = L.id2row.find(ids[r]);
        if (it == L.id2row.end()) {
            if (!insert_if_absent) {
                missing = true;
                break;
            }
            const int64_t row = L.len + (int64_t)appended.size();
            appended.push_back(r);
            L.id2row.emplace(ids[r], row);
            dst_src[row] = r;
        } else {
            dst_src[it->second] = r;
        }
    }
    const int64_t nappend = (int64_t)appended.size();
    if (nappend) ensure_list_room(ix, l, L.len + nappend);
    if (!dst_src.empty()) {
        std::vector<int64_t> dst_rows;
        std::vector<float> staging;
        std::vector<int64_t> row_ids;
        dst_rows.reserve(dst_src.size());
        staging.reserve(dst_src.size() * ix.dim);
        for (auto& kv : dst_src) {
            dst_rows.push_back(L.off + kv.first);
            staging.insert(staging.end(), vecs + kv.second * ix.dim, vecs + (kv.second + 1) * ix.dim);
            row_ids.push_back(ids[kv.second]);
        }
        const int64_t m = (int64_t)dst_rows.size();
        // the rows in the arena's format (and their norms), then scattered into place
        DBuf<float> d_src, nrm;
        d_src.alloc((size_t)(m * ix.row_bytes() / 4));
        nrm.alloc((size_t)m);
        if (ix.ldr != ix.dim || ix.bf16_rows())
            M3G_CK(cudaMemsetAsync(d_src.p, 0, (size_t)(m * ix.row_bytes()), ix.wstream));
        store_rows(ix, reinterpret_cast<unsigned char*>(d_src.p), staging.data(), m, nrm.p);
        DevIdx di, dids;
        di.upload(dst_rows, ix.wstream);
        dids.upload(row_ids, ix.wstream);
        const int w = ix.row_words();
        M3G_CK(launch_scatter_rows(d_src.p, w, di.d.p, m, w, ix.vecs.p, w, ix.wstream));
        M3G_CK(launch_scatter_i64(dids.d.p, di.d.p, m, ix.ids.p, ix.wstream));
        M3G_CK(launch_set_bytes(ix.alive.p, di.d.p, m, 1, ix.wstream));
        M3G_CK(launch_scatter_rows(nrm.p, 1, di.d.p, m, 1, ix.rnorm2.p, 1, ix.wstream));
        M3G_CK(cudaStreamSynchronize(ix.wstream));
    }
    for (int64_t i = 0; i < nappend; ++i) {
        L.ids.push_back(ids[appended[i]]);
        L.alive.push_back(1);
    }
    L.len += nappend;
    L.live += nappend;
    if (missing) fail(M3G_ERUNTIME, "Cluster::update_batch: id not found");
}

// Cluster::erase_batch (cluster.cpp:135-150).
void list_erase(Index& ix, int l, const int64_t* ids, int64_t n) {
    if (!ids || n == 0) return;
    ListMeta& L = ix.lists[l];
    std::vector<int64_t> rows;
    for (int64_t r = 0; r < n; ++r) {
        auto it = L.id2row.find(ids[r]);
        if (it == L.id2row.end()) continue;
        const int64_t row = it->second;
        if (row < (int64_t)L.alive.size() && L.alive[row]) {
            L.alive[row] = 0;
            if (L.live > 0) --L.live;
            rows.push_back(L.off + row);
        }
        L.id2row.erase(it);
    }
    if (!rows.empty()) {
        DevIdx di;
        di.upload(rows, ix.wstream);
        M3G_CK(launch_set_bytes(ix.alive.p, di.d.p, (int64_t)rows.size(), 0, ix.wstream));
        M3G_CK(cudaStreamSynchronize(ix.wstream));
    }
}

// Moves the given rows of list l (list-relative, ascending) into a fresh
// segment of list `dst_list` (which may be l itself), in that order.
void regroup_rows(Index& ix, int l, const std::vector<int64_t>& rows, int dst_list) {
    ListMeta& S = ix.lists[l];
    const int64_t n = (int64_t)rows.size();
    std::vector<int64_t> src_abs(rows.size());
    for (size_t i = 0; i < rows.size(); ++i) src_abs[i] = S.off + rows[i];
    std::vector<int64_t> new_ids(rows.size());
    for (size_t i = 0; i < rows.size(); ++i) new_ids[i] = S.ids[rows[i]];
    const int64_t cap = std::max<int64_t>(n, 16);
    if (ix.arena_used + cap > ix.arena_cap) {
        grow_arena(ix, cap);
        for (size_t i = 0; i < rows.size(); ++i) src_abs[i] = ix.lists[l].off + rows[i];
    }
    const int64_t dst = ix.arena_used;
    ix.arena_used += cap;
    if (n > 0) {
        DevIdx di;
        di.upload(src_abs, ix.wstream);
        const int w = ix.row_words();
        M3G_CK(launch_gather_rows(ix.vecs.p, w, di.d.p, n, w, reinterpret_cast<float*>(ix.row_ptr(dst)),
                                  w, ix.wstream));
        M3G_CK(launch_gather_f32(ix.rnorm2.p, di.d.p, n, ix.rnorm2.p + dst, ix.wstream));
        M3G_CK(launch_gather_i64(ix.ids.p, di.d.p, n, ix.ids.p + dst, ix.wstream));
        M3G_CK(cudaMemsetAsync(ix.alive.p + dst, 1, (size_t)n, ix.wstream));
        M3G_CK(cudaStreamSynchronize(ix.wstream));
    }
    ListMeta& D = ix.lists[dst_list];
    D.off = dst;
    D.cap = cap;
    D.len = n;
    D.live = n;
    D.ids = std::move(new_ids);
    D.alive.assign((size_t)n, 1);
    D.id2row.clear();
    for (int64_t r = 0; r < n; ++r) D.id2row.emplace(D.ids[r], r);
}

// Cluster::compact (cluster.cpp:276-309).
void list_compact(Index& ix, int l) {
    ListMeta& L = ix.lists[l];
    if (L.len == 0 || L.live == L.len) return;
    std::vector<int64_t> keep;
    keep.reserve((size_t)L.live);
    for (int64_t r = 0; r < L.len; ++r)
        if (L.alive[r]) keep.push_back(r);
    regroup_rows(ix, l, keep, l);
}

}  // namespace

// ===================== Engine =====================

Engine::Engine() {
    cudaGetDevice(&device_);
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device_) == cudaSuccess && n > 0)
        num_sms_ = n;
    else
        num_sms_ = kDefaultNsm;
    cudaGetLastError();
    if (const char* v = std::getenv("M3G_SEARCH_GRAPH")) graphs_off_ = std::string(v) == "0";
}

Engine::~Engine() {
    try {
        stop();
    } catch (...) {
    }
    DeviceGuard g(device_);
    {
        std::unique_lock lk(imu_);
        indices_.clear();
    }
    if (graph_.exec) cudaGraphExecDestroy(graph_.exec);
    graph_.exec = nullptr;
    if (ws_.stream) {
        cudaStreamSynchronize(ws_.stream);
        cudaStreamDestroy(ws_.stream);
    }
    if (ws_.done) cudaEventDestroy(ws_.done);
    if (ws_.legacy) cudaEventDestroy(ws_.legacy);
    for (auto& e : ws_.ev)
        if (e) cudaEventDestroy(e);
    ws_.Q.release();
    ws_.qn.release();
    ws_.qn2.release();
    ws_.S.release();
    ws_.probes.release();
    ws_.lcount.release();
    ws_.lstart.release();
    ws_.lcursor.release();
    ws_.n_items.release();
    ws_.item_counter.release();
    ws_.pair_q.release();
    ws_.pair_slot.release();
    ws_.items.release();
    ws_.tile_cnt.release();
    ws_.plan.release();
    ws_.part_score.release();
    ws_.part_row.release();
    ws_.out_ids.release();
    ws_.out_scores.release();
    ws_.out_counts.release();
    ws_.err.release();
    if (ws_.err_host) cudaFreeHost(ws_.err_host);
    ws_.err_host = nullptr;
    ws_.stats.release();
}

void Engine::set_device(int dev) {
    int count = 0;
    M3G_CK(cudaGetDeviceCount(&count));
    if (dev < 0 || dev >= count) fail(M3G_EINVAL, "set_device: no such CUDA device");
    std::shared_lock lk(imu_);
    if (!indices_.empty() || ws_.stream) fail(M3G_ERUNTIME, "set_device: engine already in use");
    device_ = dev;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device_) == cudaSuccess && n > 0)
        num_sms_ = n;
}

std::shared_ptr<Index> Engine::find(int index_id) const {
    std::shared_lock lk(imu_);
    auto it = indices_.find(index_id);
    return it == indices_.end() ? nullptr : it->second;
}

std::shared_ptr<Index> Engine::get(int index_id, const char* who) const {
    auto ix = find(index_id);
    if (!ix) fail(M3G_ERANGE, std::string(who) + ": index not found");
    return ix;
}

// ---------------- lifecycle: m3_async.cpp:53-105 ----------------

void Engine::start(int writers, int maint) {
    if (running_.exchange(true)) return;
    for (int i = 0; i < writers; ++i) writers_.emplace_back([this] { writer_loop(); });
    for (int i = 0; i < maint; ++i) maint_.emplace_back([this] { maintenance_loop(); });
}

void Engine::stop() {
    if (!running_.exchange(false)) return;
    {
        std::lock_guard lk(qmu_);
        q_not_empty_.notify_all();
        q_not_full_.notify_all();
    }
    {
        std::lock_guard lk(maint_mu_);
        maint_cv_.notify_all();
    }
    for (auto& t : writers_) t.join();
    writers_.clear();
    for (auto& t : maint_) t.join();
    maint_.clear();
}

// ---------------- index lifecycle ----------------

void Engine::create_ivf(int index_id, int dim, int metric, bool normalized, const float* C,
                        int64_t nlist, int storage) {
    if (dim <= 0) fail(M3G_EINVAL, "IVFIndex: dim must be > 0");
    if (storage != M3G_STORE_FP32 && storage != M3G_STORE_BF16)
        fail(M3G_EINVAL, "create_ivf: unknown storage type");
    if (metric < 0 || metric > 2) fail(M3G_EINVAL, "create_ivf: unknown metric");
    if (nlist < 0 || (nlist > 0 && !C)) fail(M3G_EINVAL, "create_ivf: centroids missing");
    if (nlist > (int64_t)INT32_MAX / 2) fail(M3G_EUNSUPPORTED, "create_ivf: too many lists");
    DeviceGuard g(device_);
    auto ix = std::make_shared<Index>();
    ix->device = device_;
    ix->dim = dim;
    ix->dpad = round_up4(dim);
    ix->storage = storage;
    ix->esize = storage == M3G_STORE_BF16 ? 2 : 4;
    ix->ldr = storage == M3G_STORE_BF16 ? std::max(64, (dim + 7) & ~7) : ix->dpad;
    ix->metric = metric;
    ix->normalized = normalized;
    M3G_CK(cudaStreamCreateWithFlags(&ix->wstream, cudaStreamNonBlocking));
    ix->centroids.assign(C, C + nlist * (int64_t)dim);
    ix->lists.resize((size_t)nlist);
    ensure_centroid_cap(*ix, (size_t)std::max<int64_t>(nlist, 1));
    upload_centroids(*ix, 0, (int)nlist);
    refresh_list_meta(*ix);
    M3G_CK(cudaStreamSynchronize(ix->wstream));
    std::shared_ptr<Index> old;
    {
        std::unique_lock lk(imu_);
        auto& slot = indices_[index_id];
        old = slot;
        slot = ix;
    }
    if (old) {
        std::unique_lock lk(old->mu);
        if (ws_.done) cudaEventSynchronize(ws_.done);
    }
}

void Engine::load_cluster_device(int index_id, int cid, const int64_t* d_ids, const void* d_vecs,
                                 int64_t n, int dtype) {
    auto ix = get(index_id, "AsyncEngine::load_cluster");
    if (n < 0 || (n > 0 && (!d_ids || !d_vecs)))
        fail(M3G_EINVAL, "AsyncEngine::load_cluster: vecs.size mismatch");
    if (dtype != M3G_F32 && dtype != M3G_BF16) fail(M3G_EINVAL, "load_cluster: unknown dtype");
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (cid < 0 || cid >= ix->nlist())
        fail(M3G_ERANGE, "IVFIndex::rebuild_cluster: invalid cluster_id");
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    list_rebuild_device(*ix, cid, d_ids, d_vecs, dtype, n);
    refresh_list_meta(*ix);
}

void Engine::load_lists_device(int index_id, const int32_t* d_assign, const int64_t* d_ids,
                               const float* d_vecs, int64_t n) {
    auto ix = get(index_id, "load_lists_device");
    if (n < 0 || (n > 0 && (!d_assign || !d_ids || !d_vecs)))
        fail(M3G_EINVAL, "load_lists_device: buffers missing");
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    const int L = ix->nlist();
    cudaStream_t st = ix->wstream;
    std::vector<int32_t> a((size_t)n);
    std::vector<int64_t> ids((size_t)n);
    if (n > 0) {
        M3G_CK(cudaMemcpyAsync(a.data(), d_assign, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
        M3G_CK(cudaMemcpyAsync(ids.data(), d_ids, (size_t)n * 8, cudaMemcpyDeviceToHost, st));
        M3G_CK(cudaStreamSynchronize(st));
    }
    // stable grouping by list: the arena is laid out list after list in ascending
    // id order, each list exactly its rows long, so sorted position j is arena row j
    std::vector<int64_t> cnt((size_t)L + 1, 0);
    for (int64_t i = 0; i < n; ++i) {
        const int c = a[(size_t)i];
        if (c >= L) fail(M3G_ERANGE, "load_lists_device: cluster id out of range");
        if (c >= 0) cnt[(size_t)c + 1]++;
    }
    for (int l = 0; l < L; ++l) cnt[(size_t)l + 1] += cnt[(size_t)l];
    const int64_t m = cnt[(size_t)L];
    std::vector<int64_t> order((size_t)m);
    {
        std::vector<int64_t> cur(cnt.begin(), cnt.end() - 1);
        for (int64_t i = 0; i < n; ++i)
            if (a[(size_t)i] >= 0) order[(size_t)cur[(size_t)a[(size_t)i]]++] = i;
    }
    for (int l = 0; l < L; ++l) {
        ListMeta& M = ix->lists[(size_t)l];
        M.off = cnt[(size_t)l];
        M.len = M.cap = M.live = cnt[(size_t)l + 1] - cnt[(size_t)l];
        M.ids.resize((size_t)M.len);
        M.alive.assign((size_t)M.len, 1);
        M.id2row.clear();
        M.id2row.reserve((size_t)M.len);
        for (int64_t r = 0; r < M.len; ++r) {
            M.ids[(size_t)r] = ids[(size_t)order[(size_t)(M.off + r)]];
            M.id2row.emplace(M.ids[(size_t)r], r);
        }
    }
    // a fresh arena of exactly m rows (it grows as inserts need)
    const int64_t cap = std::max<int64_t>(m, 1024);
    ix->vecs.alloc((size_t)(cap * ix->row_bytes() / 4));
    ix->rnorm2.alloc((size_t)cap);
    ix->ids.alloc((size_t)cap);
    ix->alive.alloc((size_t)cap);
    M3G_CK(cudaMemsetAsync(ix->vecs.p, 0, (size_t)(cap * ix->row_bytes()), st));
    M3G_CK(cudaMemsetAsync(ix->alive.p, 0, (size_t)cap, st));
    ix->arena_cap = cap;
    ix->arena_used = m;
    const int64_t chunk = std::max<int64_t>(1, (int64_t(1) << 28) / ((int64_t)ix->dpad * 4));
    DBuf<float> stage;
    DBuf<int64_t> d_order;
    stage.alloc((size_t)(std::min(chunk, std::max<int64_t>(m, 1)) * ix->dpad));
    d_order.alloc((size_t)std::max<int64_t>(m, 1));
    if (m > 0)
        M3G_CK(cudaMemcpyAsync(d_order.p, order.data(), (size_t)m * 8, cudaMemcpyHostToDevice, st));
    for (int64_t j0 = 0; j0 < m; j0 += chunk) {
        const int64_t k = std::min(chunk, m - j0);
        if (ix->dpad != ix->dim)
            M3G_CK(cudaMemsetAsync(stage.p, 0, (size_t)(k * ix->dpad) * 4, st));
        M3G_CK(launch_gather_rows(d_vecs, ix->dim, d_order.p + j0, k, ix->dim, stage.p, ix->dpad, st));
        store_staged_rows(*ix, ix->row_ptr(j0), stage.p, k, ix->rnorm2.p + j0);
        M3G_CK(launch_gather_i64(d_ids, d_order.p + j0, k, ix->ids.p + j0, st));
    }
    if (m > 0) M3G_CK(cudaMemsetAsync(ix->alive.p, 1, (size_t)m, st));
    M3G_CK(cudaStreamSynchronize(st));
    rebuild_maps(*ix);
    refresh_list_meta(*ix);
}

int Engine::storage_of(int index_id) {
    auto ix = get(index_id, "storage_of");
    return ix->storage;
}

void Engine::load_cluster(int index_id, int cid, const int64_t* ids, const float* vecs, int64_t n) {
    auto ix = get(index_id, "AsyncEngine::load_cluster");
    if (n < 0 || (n > 0 && (!ids || !vecs)))
        fail(M3G_EINVAL, "AsyncEngine::load_cluster: vecs.size mismatch");
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (cid < 0 || cid >= ix->nlist())
        fail(M3G_ERANGE, "IVFIndex::rebuild_cluster: invalid cluster_id");
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    list_rebuild(*ix, cid, ids, vecs, n);
    refresh_list_meta(*ix);
}

// ---------------- queue: m3_async.cpp:123-201, 399-467 ----------------

bool Engine::enqueue(WriteOp&& op) {
    std::unique_lock lk(qmu_);
    while (running_ && queue_.size() >= qpol_.capacity) {
        if (!qpol_.block_on_full) return false;
        q_not_full_.wait(lk);
    }
    if (!running_) return false;
    queue_.emplace_back(std::move(op));
    ++enqueued_;
    q_not_empty_.notify_one();
    return true;
}

void Engine::flush() {
    {
        std::unique_lock lk(qmu_);
        while (running_ && (!queue_.empty() || applied_.load() < enqueued_.load()))
            q_not_full_.wait(lk);
    }
    std::lock_guard lk(err_mu_);
    if (first_error_code_) {
        const int code = first_error_code_;
        const std::string msg = first_error_;
        first_error_code_ = 0;
        first_error_.clear();
        fail(code, "write failed in a writer thread: " + msg);
    }
}

void Engine::record_error(const std::string& msg, int code) {
    std::lock_guard lk(err_mu_);
    if (!first_error_code_) {
        first_error_code_ = code;
        first_error_ = msg;
    }
}

namespace {
// Positions in `ids` of the ids each list holds (a live row), in op order, for
// updates and deletes addressed to every list (cluster_id kAnyList).  Probes
// every list's id map per id, or walks every list's map once when that is less
// work.
std::vector<std::vector<int64_t>> positions_by_list(const Index& ix, const std::vector<int64_t>& ids) {
    const int L = ix.nlist();
    std::vector<std::vector<int64_t>> pos((size_t)L);
    const int64_t n = (int64_t)ids.size();
    int64_t rows = 0;
    for (const auto& m : ix.lists) rows += (int64_t)m.id2row.size();
    if ((double)n * L <= (double)rows) {
        for (int l = 0; l < L; ++l)
            for (int64_t i = 0; i < n; ++i)
                if (ix.lists[(size_t)l].id2row.count(ids[(size_t)i])) pos[(size_t)l].push_back(i);
        return pos;
    }
    std::unordered_map<int64_t, std::vector<int64_t>> at;
    for (int64_t i = 0; i < n; ++i) at[ids[(size_t)i]].push_back(i);
    for (int l = 0; l < L; ++l) {
        auto& p = pos[(size_t)l];
        for (const auto& kv : ix.lists[(size_t)l].id2row) {
            auto it = at.find(kv.first);
            if (it != at.end()) p.insert(p.end(), it->second.begin(), it->second.end());
        }
        std::sort(p.begin(), p.end());
    }
    return pos;
}
}  // namespace

void Engine::apply_run(std::vector<WriteOp>& ops, size_t b, size_t e) {
    auto ix = find(ops[b].index_id);
    if (!ix) {
        for (size_t i = b; i < e; ++i) {
            record_error("writer: index " + std::to_string(ops[i].index_id) + " not found",
                         M3G_ERANGE);
            ++applied_;
        }
        return;
    }
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    for (size_t i = b; i < e; ++i) {
        try {
            apply_locked(*ix, ops[i]);
        } catch (const Error& err) {
            record_error(err.what(), err.code);
        } catch (const std::exception& err) {
            record_error(err.what(), M3G_ERUNTIME);
        }
    }
    try {
        refresh_list_meta(*ix);
    } catch (const Error& err) {
        record_error(err.what(), err.code);
    }
    applied_ += (uint64_t)(e - b);
}

void Engine::apply_locked(Index& ixr, const WriteOp& op) {
    Index* ix = &ixr;
    const bool any_list = op.cluster_id == kAnyList && op.kind != WriteOp::kInsert &&
                          op.kind != WriteOp::kInsertRouted;
    if (op.kind == WriteOp::kInsertRouted) {
        list_add_routed(*ix, op.ids, op.vecs, op.clusters, [this](const std::string& m) {
            record_error(m, M3G_ERUNTIME);
        });
        return;
    }
    if (!any_list && (op.cluster_id < 0 || op.cluster_id >= ix->nlist())) {
        const char* w = op.kind == WriteOp::kInsert   ? "IVFIndex::add_batch: invalid cluster_id"
                        : op.kind == WriteOp::kUpdate ? "IVFIndex::update_batch: invalid cluster_id"
                                                      : "IVFIndex::erase_batch: invalid cluster_id";
        fail(M3G_ERANGE, w);
    }
    const int64_t n = (int64_t)op.ids.size();
    if (any_list) {
        const auto pos = positions_by_list(*ix, op.ids);
        std::vector<int64_t> sub_ids;
        std::vector<float> sub_vecs;
        for (int l = 0; l < ix->nlist(); ++l) {
            const auto& p = pos[(size_t)l];
            if (p.empty()) continue;
            sub_ids.clear();
            sub_vecs.clear();
            for (int64_t i : p) {
                sub_ids.push_back(op.ids[(size_t)i]);
                if (op.kind == WriteOp::kUpdate)
                    sub_vecs.insert(sub_vecs.end(), op.vecs.begin() + i * ix->dim,
                                    op.vecs.begin() + (i + 1) * ix->dim);
            }
            if (op.kind == WriteOp::kUpdate)
                list_update(*ix, l, sub_ids.data(), sub_vecs.data(), (int64_t)sub_ids.size(), false);
            else
                list_erase(*ix, l, sub_ids.data(), (int64_t)sub_ids.size());
        }
        return;
    }
    switch (op.kind) {
        case WriteOp::kInsert:
            list_add(*ix, op.cluster_id, op.ids.data(), op.vecs.data(), n);
            break;
        case WriteOp::kUpdate:
            list_update(*ix, op.cluster_id, op.ids.data(), op.vecs.data(), n, op.insert_if_absent);
            break;
        case WriteOp::kDelete:
            list_erase(*ix, op.cluster_id, op.ids.data(), n);
            break;
        default:
            break;
    }
}

void Engine::writer_loop() {
    std::vector<WriteOp> batch;
    while (running_) {
        batch.clear();
        {
            std::unique_lock lk(qmu_);
            while (queue_.empty() && running_) q_not_empty_.wait(lk);
            if (!running_) break;
            const size_t m = std::min(qpol_.pop_batch_max ? qpol_.pop_batch_max : 1, queue_.size());
            for (size_t i = 0; i < m; ++i) {
                batch.push_back(std::move(queue_.front()));
                queue_.pop_front();
            }
            q_not_full_.notify_all();
        }
        // runs of consecutive ops on one index share the lock and the metadata refresh
        for (size_t b = 0; b < batch.size();) {
            size_t e = b + 1;
            while (e < batch.size() && batch[e].index_id == batch[b].index_id) ++e;
            apply_run(batch, b, e);
            b = e;
        }
        std::lock_guard lk(qmu_);
        q_not_full_.notify_all();
    }
}

void Engine::maintenance_loop() {
    while (running_) {
        {
            std::unique_lock lk(maint_mu_);
            const double p = mpol_.period_sec > 0.0 ? mpol_.period_sec : 1.0;
            maint_cv_.wait_for(lk, std::chrono::duration<double>(p), [this] { return !running_; });
        }
        if (!running_) break;
        std::vector<int> ids;
        {
            std::shared_lock lk(imu_);
            for (auto& kv : indices_) ids.push_back(kv.first);
        }
        for (int id : ids) {
            try {
                maintenance_pass(id);
            } catch (const Error& e) {
                record_error(e.what(), e.code);
            } catch (const std::exception& e) {
                record_error(e.what(), M3G_ERUNTIME);
            }
        }
    }
}

// IVFIndex::maintenance_pass (m3_index.cpp:278-312): compact lists whose live
// fraction fell below compact_ratio; optionally split oversized lists.
void Engine::maintenance_pass(int index_id) {
    auto ix = find(index_id);
    if (!ix) return;
    std::vector<int> to_split;
    {
        DeviceGuard g(device_);
        std::unique_lock lk(ix->mu);
        if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
        bool changed = false;
        for (int l = 0; l < ix->nlist(); ++l) {
            ListMeta& L = ix->lists[l];
            if (L.len == 0) continue;
            if ((double)L.live / (double)L.len < mpol_.compact_ratio) {
                list_compact(*ix, l);
                changed = true;
            }
            if (mpol_.auto_split && mpol_.split_mean_factor <= 0 &&
                (size_t)L.live > mpol_.split_threshold)
                to_split.push_back(l);
        }
        if (changed) refresh_list_meta(*ix);
    }
    if (mpol_.auto_split && mpol_.split_mean_factor > 0) {
        split_oversized(index_id, mpol_.split_mean_factor, mpol_.split_niter, 0x5eed0000ull);
        return;
    }
    for (int l : to_split) split_cluster(index_id, l, mpol_.split_niter, 0x5eed0000ull + (uint64_t)l);
}

std::vector<int> Engine::oversized_lists(int index_id, double mean_factor) {
    auto ix = get(index_id, "split_oversized");
    std::shared_lock lk(ix->mu);
    std::vector<int> out;
    const int L = ix->nlist();
    if (L == 0) return out;
    int64_t total = 0;
    for (const auto& l : ix->lists) total += l.live;
    const double limit = mean_factor * ((double)total / (double)L);
    for (int l = 0; l < L; ++l)
        if ((double)ix->lists[(size_t)l].live > limit) out.push_back(l);
    return out;
}

int Engine::split_oversized(int index_id, double mean_factor, int niter, uint64_t seed) {
    if (!(mean_factor > 0)) fail(M3G_EINVAL, "split_oversized: mean_factor must be > 0");
    if (niter < 0) fail(M3G_EINVAL, "split_oversized: niter < 0");
    auto ix = get(index_id, "split_oversized");
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    // the lists over the limit when the pass starts (live rows > factor x the mean
    // over all lists); every one is split as split_cluster would split it, all at
    // once: one segmented 2-means over their rows, then the regrouping in
    // ascending list order, so new lists get the next ids in that order
    const int L0 = ix->nlist();
    if (L0 == 0) return 0;
    int64_t total = 0;
    for (const auto& l : ix->lists) total += l.live;
    const double limit = mean_factor * ((double)total / (double)L0);
    std::vector<int> todo;
    for (int l = 0; l < L0; ++l)
        if ((double)ix->lists[(size_t)l].live > limit) {
            list_compact(*ix, l);
            if (ix->lists[(size_t)l].len >= 2) todo.push_back(l);
        }
    if (todo.empty()) {
        refresh_list_meta(*ix);
        return 0;
    }
    const int nseg = (int)todo.size();
    const int dpad = ix->dpad;
    cudaStream_t st = ix->wstream;
    std::vector<int64_t> seg_off((size_t)nseg + 1, 0);
    for (int s = 0; s < nseg; ++s) seg_off[(size_t)s + 1] = seg_off[(size_t)s] + ix->lists[(size_t)todo[(size_t)s]].len;
    const int64_t n = seg_off[(size_t)nseg];
    // the rows as fp32 [n, dpad], segment by segment
    DBuf<float> X, C2;
    DBuf<int32_t> side, row_seg;
    DBuf<int64_t> d_off;
    X.alloc((size_t)(n * dpad));
    C2.alloc((size_t)(2 * nseg) * dpad);
    side.alloc((size_t)n);
    row_seg.alloc((size_t)n);
    for (int s = 0; s < nseg; ++s) {
        const ListMeta& M = ix->lists[(size_t)todo[(size_t)s]];
        float* dst = X.p + seg_off[(size_t)s] * dpad;
        if (ix->bf16_rows())
            M3G_CK(launch_unpack_bf16_rows(reinterpret_cast<const __nv_bfloat16*>(ix->row_ptr(M.off)),
                                           ix->ldr, M.len, ix->dim, dst, dpad, st));
        else
            M3G_CK(cudaMemcpyAsync(dst, ix->row_ptr(M.off), (size_t)(M.len * dpad) * 4,
                                   cudaMemcpyDeviceToDevice, st));
    }
    std::vector<int32_t> rs((size_t)n);
    std::vector<int64_t> init((size_t)2 * nseg);
    for (int s = 0; s < nseg; ++s) {
        const int64_t b = seg_off[(size_t)s], e = seg_off[(size_t)s + 1];
        std::fill(rs.begin() + b, rs.begin() + e, s);
        int64_t pick[2];
        sample_rows(seed + (uint64_t)todo[(size_t)s], e - b, 2, pick);
        init[(size_t)2 * s] = b + pick[0];
        init[(size_t)2 * s + 1] = b + pick[1];
    }
    M3G_CK(cudaMemcpyAsync(row_seg.p, rs.data(), (size_t)n * 4, cudaMemcpyHostToDevice, st));
    d_off.alloc((size_t)nseg + 1);
    M3G_CK(cudaMemcpyAsync(d_off.p, seg_off.data(), seg_off.size() * 8, cudaMemcpyHostToDevice, st));
    DevIdx di;
    di.upload(init, st);
    M3G_CK(launch_gather_rows(X.p, dpad, di.d.p, 2 * nseg, dpad, C2.p, dpad, st));
    const int nz = ix->normalized ? 1 : 0;
    for (int it = 0; it < niter; ++it) {
        M3G_CK(launch_seg2_assign(X.p, dpad, row_seg.p, n, C2.p, ix->dim, ix->metric, nz, side.p, st));
        M3G_CK(launch_seg2_update(X.p, dpad, d_off.p, nseg, side.p, ix->dim, C2.p, st));
    }
    M3G_CK(launch_seg2_assign(X.p, dpad, row_seg.p, n, C2.p, ix->dim, ix->metric, nz, side.p, st));
    std::vector<float> c2((size_t)(2 * nseg) * ix->dim);
    M3G_CK(cudaMemcpy2DAsync(c2.data(), (size_t)ix->dim * 4, C2.p, (size_t)dpad * 4,
                             (size_t)ix->dim * 4, (size_t)(2 * nseg), cudaMemcpyDeviceToHost, st));
    std::vector<int32_t> sd((size_t)n);
    M3G_CK(cudaMemcpyAsync(sd.data(), side.p, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    M3G_CK(cudaStreamSynchronize(st));
    // set_centroid(l, c0); add_cluster(c1); rows regrouped in list order
    // (m3_index.cpp:133-163), list by list in ascending id order
    ensure_centroid_cap(*ix, (size_t)(L0 + nseg));
    for (int s = 0; s < nseg; ++s) {
        const int l = todo[(size_t)s];
        const float* c0 = &c2[(size_t)(2 * s) * ix->dim];
        std::copy(c0, c0 + ix->dim, ix->centroids.begin() + (size_t)l * ix->dim);
        upload_centroids(*ix, l, 1);
        const int nid = ix->nlist();
        ix->centroids.insert(ix->centroids.end(), c0 + ix->dim, c0 + 2 * ix->dim);
        ix->lists.emplace_back();
        upload_centroids(*ix, nid, 1);
        std::vector<int64_t> side0, side1;
        for (int64_t r = seg_off[(size_t)s]; r < seg_off[(size_t)s + 1]; ++r)
            (sd[(size_t)r] == 1 ? side1 : side0).push_back(r - seg_off[(size_t)s]);
        regroup_rows(*ix, l, side1, nid);
        regroup_rows(*ix, l, side0, l);
    }
    refresh_list_meta(*ix);
    return nseg;
}

void Engine::compact_cluster(int index_id, int cid) {
    auto ix = find(index_id);
    if (!ix) return;
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (cid < 0 || cid >= ix->nlist()) return;
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    list_compact(*ix, cid);
    refresh_list_meta(*ix);
}

// ---------------- info ----------------

void Engine::info(int index_id, int* dim, int* metric, int* normalized, int* nlist) {
    auto ix = find(index_id);
    if (!ix) {  // m3_async.cpp:317-351 defaults
        if (dim) *dim = 0;
        if (metric) *metric = M3G_COSINE;
        if (normalized) *normalized = 1;
        if (nlist) *nlist = 0;
        return;
    }
    std::shared_lock lk(ix->mu);
    if (dim) *dim = ix->dim;
    if (metric) *metric = ix->metric;
    if (normalized) *normalized = ix->normalized ? 1 : 0;
    if (nlist) *nlist = ix->nlist();
}

void Engine::cluster_size(int index_id, int cid, int64_t* size, int64_t* live) {
    auto ix = get(index_id, "cluster_size");
    std::shared_lock lk(ix->mu);
    if (cid < 0 || cid >= ix->nlist()) fail(M3G_ERANGE, "cluster_size: invalid cluster_id");
    if (size) *size = ix->lists[cid].len;
    if (live) *live = ix->lists[cid].live;
}

void Engine::get_centroids(int index_id, float* out) {
    auto ix = get(index_id, "get_centroids");
    std::shared_lock lk(ix->mu);
    std::copy(ix->centroids.begin(), ix->centroids.end(), out);
}

namespace {
// Live rows of list `cid` of an index held under its lock: ids and vectors
// (dim floats per row) in row order.
void live_rows(Index& ix, int cid, std::vector<int64_t>* ids, std::vector<float>* vecs) {
    const ListMeta& L = ix.lists[(size_t)cid];
    ids->clear();
    vecs->clear();
    if (L.len == 0 || L.live == 0) return;
    std::vector<float> all((size_t)(L.len * ix.dim));
    M3G_CK(cudaStreamSynchronize(ix.wstream));
    if (ix.bf16_rows()) {
        // widened on the device (the bf16 values exactly), then copied out
        DBuf<float> wide;
        wide.alloc((size_t)(L.len * ix.dim));
        M3G_CK(launch_unpack_bf16_rows(reinterpret_cast<const __nv_bfloat16*>(ix.row_ptr(L.off)),
                                       ix.ldr, L.len, ix.dim, wide.p, ix.dim, ix.wstream));
        M3G_CK(cudaMemcpyAsync(all.data(), wide.p, all.size() * 4, cudaMemcpyDeviceToHost,
                               ix.wstream));
        M3G_CK(cudaStreamSynchronize(ix.wstream));
    } else {
        M3G_CK(cudaMemcpy2D(all.data(), (size_t)ix.dim * 4, ix.row_ptr(L.off), (size_t)ix.ldr * 4,
                            (size_t)ix.dim * 4, (size_t)L.len, cudaMemcpyDeviceToHost));
    }
    ids->reserve((size_t)L.live);
    vecs->reserve((size_t)(L.live * ix.dim));
    for (int64_t r = 0; r < L.len; ++r) {
        if (!L.alive[(size_t)r]) continue;
        ids->push_back(L.ids[(size_t)r]);
        vecs->insert(vecs->end(), all.begin() + r * ix.dim, all.begin() + (r + 1) * ix.dim);
    }
}

constexpr char kIndexMagic[8] = {'M', '3', 'G', 'I', 'V', 'F', '0', '1'};
// version 2 adds the list storage type (int32) after the four header fields
constexpr char kIndexMagic2[8] = {'M', '3', 'G', 'I', 'V', 'F', '0', '2'};
}  // namespace

void Engine::get_cluster(int index_id, int cid, int64_t* ids, float* vecs, int64_t cap,
                         int64_t* n_live) {
    auto ix = get(index_id, "get_cluster");
    DeviceGuard g(device_);
    std::shared_lock lk(ix->mu);
    if (cid < 0 || cid >= ix->nlist()) fail(M3G_ERANGE, "get_cluster: invalid cluster_id");
    const int64_t live = ix->lists[(size_t)cid].live;
    if (n_live) *n_live = live;
    if (!ids && !vecs) return;
    if (cap < live) fail(M3G_EINVAL, "get_cluster: output capacity below the list's live rows");
    std::vector<int64_t> i;
    std::vector<float> v;
    live_rows(*ix, cid, &i, &v);
    if (ids) std::copy(i.begin(), i.end(), ids);
    if (vecs) std::copy(v.begin(), v.end(), vecs);
}

// File layout (little-endian): 8-byte magic "M3GIVF02"; int32 dim, metric,
// normalized, nlist, storage; float centroids[nlist * dim]; then per list int64
// n, int64 ids[n], float vectors[n * dim] (the live rows, in row order; a bf16
// index's rows as their exact fp32 values).  "M3GIVF01" files (no storage
// field, fp32) still load.
void Engine::save_index(int index_id, const char* path) {
    auto ix = get(index_id, "save_index");
    if (!path) fail(M3G_EINVAL, "save_index: path missing");
    DeviceGuard g(device_);
    std::shared_lock lk(ix->mu);
    FILE* f = std::fopen(path, "wb");
    if (!f) fail(M3G_ERUNTIME, std::string("save_index: cannot open ") + path);
    bool ok = true;
    auto put = [&](const void* p, size_t bytes) {
        if (ok && bytes && std::fwrite(p, 1, bytes, f) != bytes) ok = false;
    };
    const int32_t hdr[5] = {ix->dim, ix->metric, ix->normalized ? 1 : 0, ix->nlist(), ix->storage};
    put(kIndexMagic2, sizeof(kIndexMagic2));
    put(hdr, sizeof(hdr));
    put(ix->centroids.data(), ix->centroids.size() * 4);
    std::vector<int64_t> ids;
    std::vector<float> vecs;
    for (int c = 0; c < ix->nlist() && ok; ++c) {
        live_rows(*ix, c, &ids, &vecs);
        const int64_t n = (int64_t)ids.size();
        put(&n, sizeof(n));
        put(ids.data(), ids.size() * 8);
        put(vecs.data(), vecs.size() * 4);
    }
    if (std::fclose(f) != 0) ok = false;
    if (!ok) fail(M3G_ERUNTIME, std::string("save_index: write failed: ") + path);
}

void Engine::load_index(int index_id, const char* path) {
    if (!path) fail(M3G_EINVAL, "load_index: path missing");
    FILE* f = std::fopen(path, "rb");
    if (!f) fail(M3G_ERUNTIME, std::string("load_index: cannot open ") + path);
    std::unique_ptr<FILE, int (*)(FILE*)> guard(f, std::fclose);
    auto get_bytes = [&](void* p, size_t bytes) {
        if (bytes && std::fread(p, 1, bytes, f) != bytes)
            fail(M3G_ERUNTIME, std::string("load_index: truncated file: ") + path);
    };
    char magic[8];
    get_bytes(magic, sizeof(magic));
    const bool v2 = std::memcmp(magic, kIndexMagic2, sizeof(magic)) == 0;
    if (!v2 && std::memcmp(magic, kIndexMagic, sizeof(magic)) != 0)
        fail(M3G_EINVAL, std::string("load_index: not an index file: ") + path);
    int32_t hdr[5] = {0, 0, 0, 0, M3G_STORE_FP32};
    get_bytes(hdr, (v2 ? 5 : 4) * sizeof(int32_t));
    const int dim = hdr[0], metric = hdr[1], nlist = hdr[3], storage = hdr[4];
    if (dim <= 0 || metric < 0 || metric > 2 || nlist < 0 ||
        (storage != M3G_STORE_FP32 && storage != M3G_STORE_BF16))
        fail(M3G_EINVAL, std::string("load_index: bad header: ") + path);
    std::vector<float> C((size_t)nlist * dim);
    get_bytes(C.data(), C.size() * 4);
    // every list is read before the index is replaced, so a bad file changes nothing
    std::vector<std::vector<int64_t>> ids((size_t)nlist);
    std::vector<std::vector<float>> vecs((size_t)nlist);
    for (int c = 0; c < nlist; ++c) {
        int64_t n = 0;
        get_bytes(&n, sizeof(n));
        if (n < 0 || n > (int64_t(1) << 40))
            fail(M3G_EINVAL, std::string("load_index: bad list size: ") + path);
        ids[(size_t)c].resize((size_t)n);
        vecs[(size_t)c].resize((size_t)n * dim);
        get_bytes(ids[(size_t)c].data(), (size_t)n * 8);
        get_bytes(vecs[(size_t)c].data(), (size_t)n * dim * 4);
    }
    create_ivf(index_id, dim, metric, hdr[2] != 0, C.data(), nlist, storage);
    for (int c = 0; c < nlist; ++c)
        if (!ids[(size_t)c].empty())
            load_cluster(index_id, c, ids[(size_t)c].data(), vecs[(size_t)c].data(),
                         (int64_t)ids[(size_t)c].size());
}

int Engine::add_cluster(int index_id, const float* c) {
    auto ix = get(index_id, "IVFIndex::add_cluster");
    if (!c) fail(M3G_EINVAL, "IVFIndex::add_cluster: centroid dim mismatch");
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    const int cid = ix->nlist();
    ensure_centroid_cap(*ix, (size_t)cid + 1);
    ix->centroids.insert(ix->centroids.end(), c, c + ix->dim);
    ix->lists.emplace_back();
    upload_centroids(*ix, cid, 1);
    refresh_list_meta(*ix);
    return cid;
}

void Engine::set_centroid(int index_id, int cid, const float* c) {
    auto ix = get(index_id, "IVFIndex::set_centroid");
    if (!c) fail(M3G_EINVAL, "IVFIndex::set_centroid: centroid dim mismatch");
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (cid < 0 || cid >= ix->nlist()) fail(M3G_ERANGE, "IVFIndex::set_centroid: invalid cluster_id");
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    std::copy(c, c + ix->dim, ix->centroids.begin() + (size_t)cid * ix->dim);
    upload_centroids(*ix, cid, 1);
    M3G_CK(cudaStreamSynchronize(ix->wstream));
}

// ---------------- search pipeline ----------------

namespace {
constexpr int64_t kMaxChunkQueries = 32768;
constexpr int64_t kMaxScoreEntries = int64_t(1) << 26;  // nq * L per chunk
constexpr int64_t kMaxPartEntries = int64_t(1) << 27;   // nq * P * k per chunk
constexpr int64_t kMaxAssignRows = int64_t(1) << 22;    // GEMM grid.y stays < 65536
// Partial lists of the row-tile region (tensor-core scan): as many as the
// (query, probe) pairs of a chunk, and at least kMinTilePartials.
constexpr int64_t kMinTilePartials = 16384;
int64_t tile_partials(int64_t nq, int64_t P) { return std::max(nq * P, kMinTilePartials); }
// Row tile of a long list when none is set: about this many bytes of rows.
constexpr int64_t kAutoTileBytes = int64_t(4) << 20;

float gamma_of(int D) { return (float)(D + 4) * 5.9604645e-8f * 1.01f; }
}  // namespace

// Runs one query chunk whose queries (rows of dQ, stride ldq >= dpad, zero padded)
// are on the device.  fixed_probes: if non-null, [nq, P] probe lists already on
// the device (skips the coarse step).  Outputs [nq, k] / [nq] on the device.
int Engine::scan_tile_rows(const Index& ix, int64_t pairs) const {
    if (scan_tile_rows_ < 0) return 0;
    if (scan_tile_rows_ > 0) return scan_tile_rows_;
    // fewer (query, probe) pairs than SMs: the smallest tiles, so the few lists a
    // small batch probes spread over the SMs
    if (pairs < num_sms_) return 128;
    const int64_t rows = kAutoTileBytes / std::max<int64_t>(1, ix.row_bytes());
    return (int)std::min<int64_t>(std::max<int64_t>(128, rows & ~int64_t(127)), int64_t(1) << 20);
}

void Engine::run_search(Index& ix, const float* dQ, int64_t ldq, int64_t nq, int k, int P,
                        const int32_t* fixed_probes, int64_t* d_ids, float* d_scores,
                        int32_t* d_counts, cudaStream_t st, bool profile, bool clear_partials) {
    Workspace& w = ws_;
    const int L = ix.nlist();
    const int D = ix.dim;
    cudaEvent_t* ev = w.ev;
    if (profile) M3G_CK(cudaEventRecord(ev[0], st));
    // the queries' norms and, for the tensor-core coarse GEMM, their split rows
    const bool split_q = !fixed_probes && P < L && use_tc_gemm();
    M3G_CK(launch_query_prep(dQ, ldq, nq, D, ix.dpad, gemm_tc_kdim(ix.dpad),
                             split_q ? w.Q3.p : nullptr, w.qn.p, w.qn2.p, st));
    if (profile) M3G_CK(cudaEventRecord(ev[1], st));
    const int32_t* probes = fixed_probes;
    if (!probes) {
        if (P >= L) {
            M3G_CK(launch_iota_rows(w.probes.p, nq, P, st));
            if (profile) M3G_CK(cudaEventRecord(ev[2], st));
        } else {
            const float beta = coarse_gemm(dQ, ldq, w.Q3.p, ix.C.p, ix.dpad, ix.C3.p, w.S.p, L,
                                           (int)nq, L, ix.dpad, w.err.p, st);
            if (profile) M3G_CK(cudaEventRecord(ev[2], st));
            M3G_CK(launch_select_probes(w.S.p, L, dQ, ldq, ix.C.p, ix.dpad, w.qn.p, w.qn2.p, ix.cn.p,
                                        ix.cn2.p, (int)nq, L, D, ix.metric, ix.normalized ? 1 : 0,
                                        beta, gamma_of(D), P, kSelectSetOnly, w.probes.p, st));
        }
        probes = w.probes.p;
    } else if (profile) {
        M3G_CK(cudaEventRecord(ev[2], st));
    }
    if (profile) M3G_CK(cudaEventRecord(ev[3], st));
    // bf16 rows are scanned by the tensor-core kernel only
    const bool tc_scan = (use_tc_scan() || ix.bf16_rows()) && scan_tc_supported(ix.metric, k);
    if (!tc_scan && ix.bf16_rows())
        fail(M3G_EUNSUPPORTED, "search: an index with bf16 storage serves k <= 128");
    const int gmax = tc_scan ? scan_tc_gmax(k) : scan_gmax_for_dim(ix.dpad);
    if (gmax <= 0) fail(M3G_EUNSUPPORTED, "search: dimension too large for the list scan");
    // with cleared partial lists, pairs probing empty lists (on a shard: the lists
    // other ranks own) are not queued
    // long lists are scanned in row tiles (tensor-core scan), so that their rows
    // spread over the SMs
    const int tile_rows = tc_scan ? scan_tile_rows(ix, nq * P) : 0;
    const int64_t tcap = tile_partials(nq, P);
    M3G_CK(launch_build_worklist(probes, (int)nq, P, L, ix.d_list_order.p, gmax, w.lcount.p,
                                 w.lstart.p, w.lcursor.p, w.items.p, w.n_items.p, w.pair_q.p,
                                 w.pair_slot.p, w.plan.p, st,
                                 clear_partials ? ix.d_list_len.p : nullptr,
                                 ix.d_list_len.p, tile_rows, (int)std::min<int64_t>(tcap, INT32_MAX)));
    if (tile_rows > 0) M3G_CK(cudaMemsetAsync(w.tile_cnt.p, 0, sizeof(int32_t) * (size_t)tcap, st));
    if (profile) {
        M3G_CK(cudaMemsetAsync(w.stats.p, 0, 3 * sizeof(unsigned long long), st));
        M3G_CK(launch_probed_rows(w.lcount.p, ix.d_list_len.p, L, gmax, w.stats.p, w.stats.p + 1,
                                  w.stats.p + 2, st));
        M3G_CK(cudaEventRecord(ev[4], st));
    }
    // the item counter and the per-query score bounds of the tensor-core scan
    M3G_CK(cudaMemsetAsync(w.item_counter.p, 0, sizeof(int32_t) * (size_t)(1 + nq), st));
    // probe slots the work list skips (probe -1) keep empty partial lists
    if (clear_partials)
        M3G_CK(launch_clear_partials(w.part_score.p, w.part_row.p, nq * P * k, st));
    ScanArgs a{};
    a.Q = dQ;
    a.dpad = (int)ldq;
    a.list_off = ix.d_list_off.p;
    a.list_len = ix.d_list_len.p;
    a.alive = ix.alive.p;
    a.rnorm2 = ix.rnorm2.p;
    a.qnorm2 = w.qn2.p;
    a.items = w.items.p;
    a.n_items = w.n_items.p;
    a.item_counter = w.item_counter.p;
    a.qbound = reinterpret_cast<uint32_t*>(w.item_counter.p + 1);
    a.pair_q = w.pair_q.p;
    a.pair_slot = w.pair_slot.p;
    a.k = k;
    a.P = P;
    a.metric = ix.metric;
    a.normalized = ix.normalized ? 1 : 0;
    a.part_score = w.part_score.p;
    a.part_row = w.part_row.p;
    a.err = w.err.p;
    a.test_wait_ns = test_wait_ns_;
    a.tile_base = nq * P;
    a.tile_cnt = w.tile_cnt.p;
    const int grid = (int)std::min<int64_t>(num_sms_, std::max<int64_t>(1, nq * P));
    if (ix.maps_valid) {
        if (tc_scan)
            M3G_CK(launch_list_scan_tc(ix.maps, a, ix.bf16_rows(), grid, st));
        else
            M3G_CK(launch_list_scan(ix.maps, a, gmax, grid, st));
    } else {
        // empty arena: every partial list is empty
        M3G_CK(cudaMemsetAsync(w.part_row.p, 0xff, sizeof(int64_t) * (size_t)(nq * P * k), st));
        std::vector<float> inf((size_t)(nq * P * k), INFINITY);
        M3G_CK(cudaMemcpyAsync(w.part_score.p, inf.data(), inf.size() * 4, cudaMemcpyHostToDevice, st));
        M3G_CK(cudaStreamSynchronize(st));
    }
    if (profile) M3G_CK(cudaEventRecord(ev[5], st));
    // the tensor-core scan ranks squared L2 by its expansion; the answer's rows are
    // rescored in the reference's arithmetic
    MergeRescore rs{dQ, ldq, ix.vecs.p, ix.ldr, D, ix.bf16_rows() ? 1 : 0};
    const bool rescore = tc_scan && ix.metric == M3G_L2 && ix.maps_valid;
    M3G_CK(launch_merge_topk(w.part_score.p, w.part_row.p, ix.ids.p, (int)nq, P, k, d_ids, d_scores,
                             d_counts, st, rescore ? &rs : nullptr));
    if (profile) M3G_CK(cudaEventRecord(ev[6], st));
    // kernels launched: query prep, coarse (gemm + select, or iota), 5 work-list
    // kernels, scan, merge (+ the exact rescoring for L2, + the byte counter when
    // profiling)
    int launches = 1 + (fixed_probes ? 0 : (P >= L ? 1 : 2)) + 5 +
                   (ix.maps_valid ? 1 : 0) + 1 + (rescore ? 1 : 0);
    if (profile) launches += 1;
    last_launches_ += launches;
}

std::vector<uintptr_t> Engine::graph_key(const Index& ix, int64_t nq, int k, int P) const {
    const Workspace& w = ws_;
    auto u = [](const void* p) { return reinterpret_cast<uintptr_t>(p); };
    return {u(&ix), u(ix.vecs.p), u(ix.ids.p), u(ix.alive.p), u(ix.rnorm2.p), u(ix.C.p),
            u(ix.C3.p), u(ix.cn.p), u(ix.cn2.p), u(ix.d_list_off.p), u(ix.d_list_len.p),
            u(ix.d_list_order.p), (uintptr_t)ix.arena_cap, (uintptr_t)ix.nlist(),
            (uintptr_t)ix.dim, (uintptr_t)ix.dpad, (uintptr_t)ix.ldr, (uintptr_t)ix.esize,
            (uintptr_t)ix.metric,
            (uintptr_t)ix.normalized, (uintptr_t)ix.maps_valid, (uintptr_t)nq, (uintptr_t)k,
            (uintptr_t)P, u(w.Q.p), u(w.Q3.p), u(w.S.p), u(w.qn.p), u(w.qn2.p), u(w.probes.p),
            u(w.lcount.p), u(w.lstart.p), u(w.lcursor.p), u(w.items.p), u(w.n_items.p),
            u(w.item_counter.p), u(w.pair_q.p), u(w.pair_slot.p), u(w.plan.p), u(w.part_score.p),
            u(w.part_row.p), u(w.out_ids.p), u(w.out_scores.p), u(w.out_counts.p), u(w.err.p),
            (uintptr_t)use_tc_scan(), (uintptr_t)use_tc_gemm(), (uintptr_t)test_wait_ns_,
            (uintptr_t)(intptr_t)scan_tile_rows(ix, nq * P), u(w.tile_cnt.p)};
}

// Replays (capturing first when the key changed) run_search on ws_.Q into
// ws_.out_* on stream st.  False when graphs are off or a capture failed (the
// caller then runs the kernels directly).
bool Engine::run_search_graph(Index& ix, int64_t nq, int k, int P, cudaStream_t st) {
    if (graphs_off_) return false;
    auto key = graph_key(ix, nq, k, P);
    for (const auto& f : graph_failed_)
        if (f == key) return false;
    if (!graph_.exec || graph_.key != key) {
        if (graph_.exec) cudaGraphExecDestroy(graph_.exec);
        graph_.exec = nullptr;
        graph_.key.clear();
        // captured on the engine's own stream (a caller's stream may be the legacy
        // default stream, which cannot be captured); launched on the caller's
        const int32_t launches = last_launches_;
        cudaGraph_t g = nullptr;
        bool ok = cudaStreamBeginCapture(ws_.stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
        if (ok) {
            try {
                run_search(ix, ws_.Q.p, ix.dpad, nq, k, P, nullptr, ws_.out_ids.p,
                           ws_.out_scores.p, ws_.out_counts.p, ws_.stream, false);
            } catch (...) {
                ok = false;
            }
            if (cudaStreamEndCapture(ws_.stream, &g) != cudaSuccess) ok = false;
        }
        if (ok && g) ok = cudaGraphInstantiate(&graph_.exec, g, 0) == cudaSuccess;
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();  // a failed capture leaves no error behind
        if (!ok || !graph_.exec) {
            // this shape runs its kernels directly from now on; other shapes keep
            // their graphs (the failure is counted in m3g_last_profile)
            graph_.exec = nullptr;
            if (graph_failed_.size() >= 64) graph_failed_.erase(graph_failed_.begin());
            graph_failed_.push_back(std::move(key));
            ++graph_failures_;
            last_launches_ = launches;
            return false;
        }
        graph_.key = std::move(key);
    } else {
        // the kernels a replay runs, for the caller's accounting
        const bool tc = (use_tc_scan() || ix.bf16_rows()) && scan_tc_supported(ix.metric, k);
        last_launches_ += 1 + (P >= ix.nlist() ? 1 : 2) + 5 + (ix.maps_valid ? 1 : 0) + 1 +
                          (tc && ix.metric == M3G_L2 && ix.maps_valid ? 1 : 0);
    }
    M3G_CK(cudaGraphLaunch(graph_.exec, st));
    ++graph_launches_;
    return true;
}

namespace {
struct WsSizes {
    int64_t nq, L, P, k, dpad;
    bool scores;  // the coarse step's score matrix and split queries are needed
};
template <class T>
bool short_of(const DBuf<T>& b, int64_t n) {
    return (size_t)n > b.n;
}
bool ws_needs_grow(const Workspace& w, const WsSizes& s) {
    const int64_t np = s.nq * s.P, nt = tile_partials(s.nq, s.P);
    return !w.err.p || short_of(w.Q, s.nq * s.dpad) || short_of(w.qn, s.nq) ||
           short_of(w.S, s.scores ? s.nq * s.L : 0) || short_of(w.probes, np) ||
           short_of(w.lcount, s.L) ||
           short_of(w.lstart, s.L) || short_of(w.lcursor, s.L) || short_of(w.plan, 6 * s.L) ||
           short_of(w.pair_q, np) ||
           short_of(w.pair_slot, np) || short_of(w.items, np + nt) || short_of(w.tile_cnt, nt) ||
           short_of(w.part_score, (np + nt) * s.k) || short_of(w.part_row, (np + nt) * s.k) ||
           short_of(w.out_ids, s.nq * s.k) || short_of(w.out_scores, s.nq * s.k) ||
           short_of(w.out_counts, s.nq) ||
           short_of(w.Q3, s.scores ? s.nq * gemm_tc_kdim((int)s.dpad) : 0) ||
           short_of(w.item_counter, 1 + s.nq);
}
void ensure_ws(Workspace& w, const WsSizes& s) {
    if (!w.err.p) {
        w.err.alloc(1);
        M3G_CK(cudaMemset(w.err.p, 0, sizeof(int)));
        if (!w.err_host) M3G_CK(cudaMallocHost(&w.err_host, sizeof(int)));
        w.stats.alloc(3);
        w.n_items.alloc(1);
    }
    w.item_counter.ensure((size_t)(1 + s.nq));
    w.Q.ensure((size_t)(s.nq * s.dpad));
    w.qn.ensure((size_t)s.nq);
    w.qn2.ensure((size_t)s.nq);
    if (s.scores) w.S.ensure((size_t)(s.nq * s.L));
    w.probes.ensure((size_t)(s.nq * s.P));
    w.lcount.ensure((size_t)s.L);
    w.lstart.ensure((size_t)s.L);
    w.lcursor.ensure((size_t)s.L);
    w.plan.ensure((size_t)(6 * s.L));
    w.pair_q.ensure((size_t)(s.nq * s.P));
    w.pair_slot.ensure((size_t)(s.nq * s.P));
    const int64_t nt = tile_partials(s.nq, s.P);
    w.items.ensure((size_t)(s.nq * s.P + nt));
    w.tile_cnt.ensure((size_t)nt);
    w.part_score.ensure((size_t)((s.nq * s.P + nt) * s.k));
    w.part_row.ensure((size_t)((s.nq * s.P + nt) * s.k));
    w.out_ids.ensure((size_t)(s.nq * s.k));
    w.out_scores.ensure((size_t)(s.nq * s.k));
    w.out_counts.ensure((size_t)s.nq);
    if (s.scores) w.Q3.ensure((size_t)(s.nq * gemm_tc_kdim((int)s.dpad)));
}

// Queries per chunk of a call.  A list probed by queries of several chunks is
// streamed once per chunk, so the chunks are as large as the buffers allow; the
// score matrix's limit applies only to calls that run the coarse step (scores).
int64_t chunk_queries(int64_t nq, int L, int P, int k, bool scores = true) {
    int64_t c = std::min<int64_t>(nq, kMaxChunkQueries);
    if (scores) c = std::min<int64_t>(c, std::max<int64_t>(1, kMaxScoreEntries / std::max(L, 1)));
    c = std::min<int64_t>(c, std::max<int64_t>(1, kMaxPartEntries / std::max<int64_t>(1, (int64_t)P * k)));
    return std::max<int64_t>(c, 1);
}
}  // namespace

void Engine::acquire_ws(cudaStream_t st, int64_t nq, int64_t L, int64_t P, int64_t k,
                        int64_t dpad, bool scores) {
    if (!ws_.stream) {
        M3G_CK(cudaStreamCreateWithFlags(&ws_.stream, cudaStreamNonBlocking));
        M3G_CK(cudaEventCreateWithFlags(&ws_.done, cudaEventDisableTiming));
        for (auto& e : ws_.ev) M3G_CK(cudaEventCreate(&e));
        M3G_CK(cudaEventRecord(ws_.done, ws_.stream));
    }
    if (!st) {
        // a call without a stream may read device data the caller produced on the
        // legacy default stream (torch's default stream, for one): the engine's own
        // stream starts after that work
        if (!ws_.legacy) M3G_CK(cudaEventCreateWithFlags(&ws_.legacy, cudaEventDisableTiming));
        M3G_CK(cudaEventRecord(ws_.legacy, cudaStreamLegacy));
        M3G_CK(cudaStreamWaitEvent(ws_.stream, ws_.legacy, 0));
        st = ws_.stream;
    }
    const WsSizes sz{nq, L, P, k, dpad, scores};
    if (ws_needs_grow(ws_, sz)) {
        M3G_CK(cudaEventSynchronize(ws_.done));
        ensure_ws(ws_, sz);
    } else if (st != ws_.last_stream) {
        M3G_CK(cudaStreamWaitEvent(st, ws_.done, 0));
    }
    ws_.last_stream = st;
}

void Engine::search(int index_id, const float* Q, int64_t nq, int k, int nprobe, bool q_dev,
                    int64_t* out_ids, float* out_scores, int32_t* out_counts, bool out_dev,
                    cudaStream_t ext_stream) {
    if (nq < 0) fail(M3G_EINVAL, "search: nq < 0");
    auto ix = find(index_id);
    DeviceGuard g(device_);
    // m3_async.cpp:224 then m3_index.cpp:372-388
    int use_nprobe = nprobe > 0 ? nprobe : spol_.default_nprobe;
    auto write_empty = [&](int64_t n) {
        if (n <= 0 || k <= 0) {
            if (n > 0) {
                if (out_dev) M3G_CK(cudaMemsetAsync(out_counts, 0, n * 4, ext_stream));
                else std::fill(out_counts, out_counts + n, 0);
            }
            return;
        }
        std::vector<int64_t> ids((size_t)(n * k), -1);
        std::vector<float> sc((size_t)(n * k), INFINITY);
        std::vector<int32_t> cn((size_t)n, 0);
        if (out_dev) {
            M3G_CK(cudaMemcpyAsync(out_ids, ids.data(), ids.size() * 8, cudaMemcpyHostToDevice, ext_stream));
            M3G_CK(cudaMemcpyAsync(out_scores, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice, ext_stream));
            M3G_CK(cudaMemcpyAsync(out_counts, cn.data(), cn.size() * 4, cudaMemcpyHostToDevice, ext_stream));
            M3G_CK(cudaStreamSynchronize(ext_stream));
        } else {
            std::copy(ids.begin(), ids.end(), out_ids);
            std::copy(sc.begin(), sc.end(), out_scores);
            std::copy(cn.begin(), cn.end(), out_counts);
        }
    };
    if (!ix || nq == 0 || k <= 0) {
        write_empty(nq);
        return;
    }
    if (!Q) fail(M3G_EINVAL, "search: queries missing");
    if (k > scan_kmax())
        fail(M3G_EUNSUPPORTED, "search: k > " + std::to_string(scan_kmax()) + " is not supported");
    std::shared_lock lk(ix->mu);
    const int L = ix->nlist();
    if (L == 0) {
        write_empty(nq);
        return;
    }
    if (use_nprobe <= 0) use_nprobe = L;
    const int P = std::min(use_nprobe, L);
    const int64_t ch = chunk_queries(nq, L, P, k);
    std::lock_guard wl(ws_.mu);
    acquire_ws(ext_stream, ch, L, P, k, ix->dpad);
    cudaStream_t st = ext_stream ? ext_stream : ws_.stream;
    const bool profile = profiling_.load() && !ext_stream;
    last_launches_ = 0;
    const bool direct_q = q_dev && ix->dpad == ix->dim && (reinterpret_cast<uintptr_t>(Q) & 15u) == 0;
    for (int64_t q0 = 0; q0 < nq; q0 += ch) {
        const int64_t m = std::min(ch, nq - q0);
        // one chunk without stage events: replayed as a CUDA graph (queries staged
        // in ws_.Q, answers copied out of ws_.out_*)
        const bool graph = m == nq && !profile && ix->maps_valid && !graphs_off_;
        const float* dQ;
        if (direct_q && !graph) {
            dQ = Q + q0 * ix->dim;
        } else if (direct_q) {
            M3G_CK(cudaMemcpyAsync(ws_.Q.p, Q + q0 * ix->dim, (size_t)(m * ix->dim) * 4,
                                   cudaMemcpyDeviceToDevice, st));
            dQ = ws_.Q.p;
        } else {
            const cudaMemcpyKind kind = q_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
            if (ix->dpad != ix->dim) {
                M3G_CK(cudaMemsetAsync(ws_.Q.p, 0, (size_t)(m * ix->dpad) * 4, st));
                M3G_CK(cudaMemcpy2DAsync(ws_.Q.p, (size_t)ix->dpad * 4, Q + q0 * ix->dim,
                                         (size_t)ix->dim * 4, (size_t)ix->dim * 4, (size_t)m, kind,
                                         st));
            } else {
                M3G_CK(cudaMemcpyAsync(ws_.Q.p, Q + q0 * ix->dim, (size_t)(m * ix->dim) * 4, kind,
                                       st));
            }
            dQ = ws_.Q.p;
        }
        if (graph && run_search_graph(*ix, m, k, P, st)) {
            const cudaMemcpyKind kind = out_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
            M3G_CK(cudaMemcpyAsync(out_ids + q0 * k, ws_.out_ids.p, (size_t)(m * k) * 8, kind, st));
            M3G_CK(cudaMemcpyAsync(out_scores + q0 * k, ws_.out_scores.p, (size_t)(m * k) * 4, kind, st));
            M3G_CK(cudaMemcpyAsync(out_counts + q0, ws_.out_counts.p, (size_t)m * 4, kind, st));
            continue;
        }
        int64_t* oi = out_dev ? out_ids + q0 * k : ws_.out_ids.p;
        float* os = out_dev ? out_scores + q0 * k : ws_.out_scores.p;
        int32_t* oc = out_dev ? out_counts + q0 : ws_.out_counts.p;
        run_search(*ix, dQ, ix->dpad, m, k, P, nullptr, oi, os, oc, st, profile && q0 == 0 && m == nq);
        if (!out_dev) {
            M3G_CK(cudaMemcpyAsync(out_ids + q0 * k, oi, (size_t)(m * k) * 8, cudaMemcpyDeviceToHost, st));
            M3G_CK(cudaMemcpyAsync(out_scores + q0 * k, os, (size_t)(m * k) * 4, cudaMemcpyDeviceToHost, st));
            M3G_CK(cudaMemcpyAsync(out_counts + q0, oc, (size_t)m * 4, cudaMemcpyDeviceToHost, st));
        }
    }
    M3G_CK(cudaEventRecord(ws_.done, st));
    if (profile) {
        prof_pending_ = true;
        prof_.kernel_launches = last_launches_;
        prof_row_bytes_ = (int64_t)ix->dim * ix->esize;  // algorithmic bytes of a stored row
        prof_dim_ = ix->dim;
        prof_.nq = (int32_t)nq;
        prof_.nprobe = P;
        prof_.k = k;
    }
    if (!ext_stream) {
        // the error flag comes back with the results: one round trip per call
        M3G_CK(cudaMemcpyAsync(ws_.err_host, ws_.err.p, sizeof(int), cudaMemcpyDeviceToHost, st));
        M3G_CK(cudaStreamSynchronize(st));
        const int err = *ws_.err_host;
        if (err) {
            M3G_CK(cudaMemset(ws_.err.p, 0, sizeof(int)));
            fail(M3G_ETIMEOUT, "search: a device-side wait gave up (kernel error " + std::to_string(err) + ")");
        }
    }
}

void Engine::sync_errors() {
    DeviceGuard g(device_);
    std::lock_guard wl(ws_.mu);
    if (!ws_.stream) return;
    M3G_CK(cudaEventSynchronize(ws_.done));
    int err = 0;
    M3G_CK(cudaMemcpy(&err, ws_.err.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) {
        M3G_CK(cudaMemset(ws_.err.p, 0, sizeof(int)));
        fail(M3G_ETIMEOUT, "search: a device-side wait gave up (kernel error " + std::to_string(err) + ")");
    }
}

m3g_profile Engine::last_profile() {
    DeviceGuard g(device_);
    std::lock_guard wl(ws_.mu);
    prof_.graph_launches = graph_launches_;
    prof_.graph_capture_failures = graph_failures_;
    if (!prof_pending_) return prof_;
    M3G_CK(cudaEventSynchronize(ws_.done));
    float t[6];
    for (int i = 0; i < 6; ++i) M3G_CK(cudaEventElapsedTime(&t[i], ws_.ev[i], ws_.ev[i + 1]));
    prof_.ms_prep = t[0];
    prof_.ms_coarse_gemm = t[1];
    prof_.ms_select = t[2];
    prof_.ms_worklist = t[3];
    prof_.ms_scan = t[4];
    prof_.ms_merge = t[5];
    M3G_CK(cudaEventElapsedTime(&prof_.ms_total, ws_.ev[0], ws_.ev[6]));
    unsigned long long st[3];
    M3G_CK(cudaMemcpy(st, ws_.stats.p, sizeof(st), cudaMemcpyDeviceToHost));
    // algorithmic bytes: every probed list read once, the queries, the results
    prof_.scan_bytes = (int64_t)st[0] * prof_row_bytes_ + (int64_t)prof_.nq * prof_dim_ * 4 +
                       (int64_t)prof_.nq * prof_.k * 12;
    prof_.probed_pairs = (int64_t)st[1];
    prof_.streamed_bytes = (int64_t)st[2] * prof_row_bytes_;
    prof_pending_ = false;
    return prof_;
}

void Engine::search_on(int index_id, const int32_t* cids, int ncids, const float* Q, int64_t nq,
                       int k, int64_t* out_ids, float* out_scores, int32_t* out_counts) {
    auto ix = find(index_id);
    DeviceGuard g(device_);
    if (!ix || nq <= 0 || k <= 0 || ncids <= 0) {
        for (int64_t i = 0; i < nq; ++i) {
            out_counts[i] = 0;
            for (int j = 0; j < k; ++j) {
                out_ids[i * k + j] = -1;
                out_scores[i * k + j] = INFINITY;
            }
        }
        return;
    }
    if (k > scan_kmax())
        fail(M3G_EUNSUPPORTED, "search_on: k > " + std::to_string(scan_kmax()) + " is not supported");
    std::shared_lock lk(ix->mu);
    const int L = ix->nlist();
    std::vector<int32_t> keep;  // m3_index.cpp:338-341: out-of-range ids are skipped
    for (int i = 0; i < ncids; ++i)
        if (cids[i] >= 0 && cids[i] < L) keep.push_back(cids[i]);
    if (keep.empty()) {
        for (int64_t i = 0; i < nq; ++i) {
            out_counts[i] = 0;
            for (int j = 0; j < k; ++j) {
                out_ids[i * k + j] = -1;
                out_scores[i * k + j] = INFINITY;
            }
        }
        return;
    }
    const int P = (int)keep.size();
    const int64_t ch = chunk_queries(nq, L, P, k, false);
    std::lock_guard wl(ws_.mu);
    acquire_ws(nullptr, ch, L, P, k, ix->dpad, false);
    cudaStream_t st = ws_.stream;
    DBuf<int32_t> row;
    row.alloc((size_t)P);
    M3G_CK(cudaMemcpyAsync(row.p, keep.data(), (size_t)P * 4, cudaMemcpyHostToDevice, st));
    for (int64_t q0 = 0; q0 < nq; q0 += ch) {
        const int64_t m = std::min(ch, nq - q0);
        if (ix->dpad != ix->dim) M3G_CK(cudaMemsetAsync(ws_.Q.p, 0, (size_t)(m * ix->dpad) * 4, st));
        M3G_CK(cudaMemcpy2DAsync(ws_.Q.p, (size_t)ix->dpad * 4, Q + q0 * ix->dim, (size_t)ix->dim * 4,
                                 (size_t)ix->dim * 4, (size_t)m, cudaMemcpyHostToDevice, st));
        M3G_CK(launch_broadcast_row(row.p, P, m, ws_.probes.p, st));
        run_search(*ix, ws_.Q.p, ix->dpad, m, k, P, ws_.probes.p, ws_.out_ids.p, ws_.out_scores.p,
                   ws_.out_counts.p, st, false);
        M3G_CK(cudaMemcpyAsync(out_ids + q0 * k, ws_.out_ids.p, (size_t)(m * k) * 8, cudaMemcpyDeviceToHost, st));
        M3G_CK(cudaMemcpyAsync(out_scores + q0 * k, ws_.out_scores.p, (size_t)(m * k) * 4, cudaMemcpyDeviceToHost, st));
        M3G_CK(cudaMemcpyAsync(out_counts + q0, ws_.out_counts.p, (size_t)m * 4, cudaMemcpyDeviceToHost, st));
    }
    M3G_CK(cudaEventRecord(ws_.done, st));
    M3G_CK(cudaStreamSynchronize(st));
    int err = 0;
    M3G_CK(cudaMemcpy(&err, ws_.err.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) {
        M3G_CK(cudaMemset(ws_.err.p, 0, sizeof(int)));
        fail(M3G_ETIMEOUT, "search_on: a device-side wait gave up");
    }
}

void Engine::select_probes(int index_id, const float* Q, int64_t nq, int nprobe, int32_t* out) {
    auto ix = get(index_id, "select_probes");
    DeviceGuard g(device_);
    std::shared_lock lk(ix->mu);
    const int L = ix->nlist();
    if (nq <= 0 || L == 0 || nprobe == 0) return;
    const int P = nprobe < 0 ? L : std::min(nprobe, L);
    const int64_t ch = chunk_queries(nq, L, P, 1);
    std::lock_guard wl(ws_.mu);
    acquire_ws(nullptr, ch, L, P, 1, ix->dpad);
    cudaStream_t st = ws_.stream;
    for (int64_t q0 = 0; q0 < nq; q0 += ch) {
        const int64_t m = std::min(ch, nq - q0);
        if (ix->dpad != ix->dim) M3G_CK(cudaMemsetAsync(ws_.Q.p, 0, (size_t)(m * ix->dpad) * 4, st));
        M3G_CK(cudaMemcpy2DAsync(ws_.Q.p, (size_t)ix->dpad * 4, Q + q0 * ix->dim, (size_t)ix->dim * 4,
                                 (size_t)ix->dim * 4, (size_t)m, cudaMemcpyHostToDevice, st));
        M3G_CK(launch_query_prep(ws_.Q.p, ix->dpad, m, ix->dim, ix->dpad, gemm_tc_kdim(ix->dpad),
                                 P < L && use_tc_gemm() ? ws_.Q3.p : nullptr, ws_.qn.p,
                                 ws_.qn2.p, st));
        if (P >= L) {
            M3G_CK(launch_iota_rows(ws_.probes.p, m, P, st));
        } else {
            const float beta = coarse_gemm(ws_.Q.p, ix->dpad, ws_.Q3.p, ix->C.p, ix->dpad,
                                           ix->C3.p, ws_.S.p, L, (int)m, L, ix->dpad, ws_.err.p,
                                           st);
            M3G_CK(launch_select_probes(ws_.S.p, L, ws_.Q.p, ix->dpad, ix->C.p, ix->dpad, ws_.qn.p,
                                        ws_.qn2.p, ix->cn.p, ix->cn2.p, (int)m, L, ix->dim,
                                        ix->metric, ix->normalized ? 1 : 0, beta,
                                        gamma_of(ix->dim), P, 0, ws_.probes.p, st));
        }
        M3G_CK(cudaMemcpyAsync(out + q0 * P, ws_.probes.p, (size_t)(m * P) * 4, cudaMemcpyDeviceToHost, st));
    }
    M3G_CK(cudaEventRecord(ws_.done, st));
    M3G_CK(cudaStreamSynchronize(st));
}

const float* Engine::stage_queries(const Index& ix, const float* dQ, int64_t m, cudaStream_t st) {
    if (ix.dpad == ix.dim && (reinterpret_cast<uintptr_t>(dQ) & 15u) == 0) return dQ;
    if (ix.dpad != ix.dim) M3G_CK(cudaMemsetAsync(ws_.Q.p, 0, (size_t)(m * ix.dpad) * 4, st));
    M3G_CK(cudaMemcpy2DAsync(ws_.Q.p, (size_t)ix.dpad * 4, dQ, (size_t)ix.dim * 4,
                             (size_t)ix.dim * 4, (size_t)m, cudaMemcpyDeviceToDevice, st));
    return ws_.Q.p;
}

void Engine::select_probes_device(int index_id, const float* dQ, int64_t nq, int nprobe,
                                  int32_t* d_out, cudaStream_t ext, bool set_only) {
    auto ix = get(index_id, "select_probes_device");
    DeviceGuard g(device_);
    std::shared_lock lk(ix->mu);
    const int L = ix->nlist();
    if (nq <= 0 || L == 0 || nprobe == 0) return;
    if (!dQ || !d_out) fail(M3G_EINVAL, "select_probes_device: buffers missing");
    const int P = nprobe < 0 ? L : std::min(nprobe, L);
    const int64_t ch = chunk_queries(nq, L, P, 1);
    std::lock_guard wl(ws_.mu);
    acquire_ws(ext, ch, L, P, 1, ix->dpad);
    cudaStream_t st = ext ? ext : ws_.stream;
    for (int64_t q0 = 0; q0 < nq; q0 += ch) {
        const int64_t m = std::min(ch, nq - q0);
        const float* q = stage_queries(*ix, dQ + q0 * ix->dim, m, st);
        int32_t* out = d_out + q0 * P;
        M3G_CK(launch_query_prep(q, ix->dpad, m, ix->dim, ix->dpad, gemm_tc_kdim(ix->dpad),
                                 P < L && use_tc_gemm() ? ws_.Q3.p : nullptr, ws_.qn.p,
                                 ws_.qn2.p, st));
        if (P >= L) {
            M3G_CK(launch_iota_rows(out, m, P, st));
        } else {
            const float beta = coarse_gemm(q, ix->dpad, ws_.Q3.p, ix->C.p, ix->dpad, ix->C3.p,
                                           ws_.S.p, L, (int)m, L, ix->dpad, ws_.err.p, st);
            M3G_CK(launch_select_probes(ws_.S.p, L, q, ix->dpad, ix->C.p, ix->dpad, ws_.qn.p,
                                        ws_.qn2.p, ix->cn.p, ix->cn2.p, (int)m, L, ix->dim,
                                        ix->metric, ix->normalized ? 1 : 0, beta,
                                        gamma_of(ix->dim), P, set_only ? kSelectSetOnly : 0, out,
                                        st));
        }
    }
    M3G_CK(cudaEventRecord(ws_.done, st));
    if (!ext) M3G_CK(cudaStreamSynchronize(st));
}

void Engine::probe_scores_device(int index_id, const float* dQ, int64_t nq,
                                 const int32_t* d_probes, int P, float* d_scores,
                                 cudaStream_t ext) {
    auto ix = get(index_id, "probe_scores_device");
    DeviceGuard g(device_);
    std::shared_lock lk(ix->mu);
    if (nq <= 0 || P <= 0) return;
    if (!dQ || !d_probes || !d_scores) fail(M3G_EINVAL, "probe_scores_device: buffers missing");
    if (ix->dim > select_max_dim()) fail(M3G_EUNSUPPORTED, "probe_scores_device: dim too large");
    const int L = ix->nlist();
    const int64_t ch = chunk_queries(nq, std::max(L, 1), P, 1, false);
    std::lock_guard wl(ws_.mu);
    acquire_ws(ext, ch, std::max(L, 1), P, 1, ix->dpad, false);
    cudaStream_t st = ext ? ext : ws_.stream;
    for (int64_t q0 = 0; q0 < nq; q0 += ch) {
        const int64_t m = std::min(ch, nq - q0);
        const float* q = stage_queries(*ix, dQ + q0 * ix->dim, m, st);
        M3G_CK(launch_probe_scores(q, ix->dpad, ix->C.p, ix->dpad, L, d_probes + q0 * P, m, P,
                                   ix->dim, ix->metric, ix->normalized ? 1 : 0, d_scores + q0 * P,
                                   st));
    }
    M3G_CK(cudaEventRecord(ws_.done, st));
    if (!ext) M3G_CK(cudaStreamSynchronize(st));
}

void Engine::search_probes_device(int index_id, const float* dQ, int64_t nq, int k,
                                  const int32_t* d_probes, int P, int64_t* d_ids, float* d_scores,
                                  int32_t* d_counts, cudaStream_t ext) {
    auto ix = get(index_id, "search_probes_device");
    DeviceGuard g(device_);
    if (nq <= 0) return;
    if (k <= 0 || P <= 0) fail(M3G_EINVAL, "search_probes_device: k and P must be positive");
    if (k > scan_kmax())
        fail(M3G_EUNSUPPORTED,
             "search_probes_device: k > " + std::to_string(scan_kmax()) + " is not supported");
    if (!dQ || !d_probes || !d_ids || !d_scores || !d_counts)
        fail(M3G_EINVAL, "search_probes_device: buffers missing");
    std::shared_lock lk(ix->mu);
    const int L = std::max(ix->nlist(), 1);
    const int64_t ch = chunk_queries(nq, L, P, k, false);
    std::lock_guard wl(ws_.mu);
    acquire_ws(ext, ch, L, P, k, ix->dpad, false);
    cudaStream_t st = ext ? ext : ws_.stream;
    for (int64_t q0 = 0; q0 < nq; q0 += ch) {
        const int64_t m = std::min(ch, nq - q0);
        const float* q = stage_queries(*ix, dQ + q0 * ix->dim, m, st);
        run_search(*ix, q, ix->dpad, m, k, P, d_probes + q0 * P, d_ids + q0 * k,
                   d_scores + q0 * k, d_counts + q0, st, false, true);
    }
    M3G_CK(cudaEventRecord(ws_.done, st));
    if (!ext) M3G_CK(cudaStreamSynchronize(st));
}

// Exact nearest-centroid assignment of n device rows (P = 1 selection).
void Engine::assign_rows(Index& ix, const float* dX, int64_t ld, const float* xn, const float* xn2,
                         int64_t n, int32_t* d_out, cudaStream_t st) {
    const int L = ix.nlist();
    const int64_t ch = std::max<int64_t>(
        1, std::min<int64_t>({n, kMaxScoreEntries / std::max(L, 1), kMaxAssignRows}));
    DBuf<float> S;
    DBuf<__nv_bfloat16> X3;
    DBuf<int> err;
    err.alloc(1);
    M3G_CK(cudaMemsetAsync(err.p, 0, sizeof(int), st));
    const int kp = gemm_tc_kdim(ix.dpad);
    S.alloc((size_t)(std::min(ch, n) * L));
    if (use_tc_gemm()) X3.alloc((size_t)(std::min(ch, n) * kp));
    for (int64_t r0 = 0; r0 < n; r0 += ch) {
        const int64_t m = std::min(ch, n - r0);
        if (use_tc_gemm())
            M3G_CK(launch_split3(dX + r0 * ld, ld, m, ix.dpad, kp, X3.p, false, st));
        const float beta = coarse_gemm(dX + r0 * ld, ld, X3.p, ix.C.p, ix.dpad, ix.C3.p, S.p, L,
                                       (int)m, L, ix.dpad, err.p, st);
        M3G_CK(launch_select_probes(S.p, L, dX + r0 * ld, ld, ix.C.p, ix.dpad, xn + r0, xn2 + r0,
                                    ix.cn.p, ix.cn2.p, (int)m, L, ix.dim, ix.metric,
                                    ix.normalized ? 1 : 0, beta, gamma_of(ix.dim), 1, 1,
                                    d_out + r0, st));
    }
    M3G_CK(cudaStreamSynchronize(st));
    int herr = 0;
    M3G_CK(cudaMemcpy(&herr, err.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) fail(M3G_ETIMEOUT, "assignment: a device-side wait gave up");
}

void Engine::nearest_clusters(int index_id, const float* vecs, int64_t n, int32_t* out,
                              bool on_device) {
    auto ix = get(index_id, "nearest_clusters");
    DeviceGuard g(device_);
    if (n <= 0) return;
    std::shared_lock lk(ix->mu);
    const int L = ix->nlist();
    if (L == 0) {
        if (on_device) M3G_CK(cudaMemset(out, 0xff, (size_t)n * 4));
        else std::fill(out, out + n, -1);
        return;
    }
    cudaStream_t st;
    M3G_CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    struct StreamGuard {
        cudaStream_t s;
        ~StreamGuard() { cudaStreamDestroy(s); }
    } sg{st};
    DBuf<float> X, xn, xn2;
    DBuf<int32_t> a;
    X.alloc((size_t)(n * ix->dpad));
    xn.alloc((size_t)n);
    xn2.alloc((size_t)n);
    a.alloc((size_t)n);
    if (ix->dpad != ix->dim) M3G_CK(cudaMemsetAsync(X.p, 0, (size_t)(n * ix->dpad) * 4, st));
    M3G_CK(cudaMemcpy2DAsync(X.p, (size_t)ix->dpad * 4, vecs, (size_t)ix->dim * 4,
                             (size_t)ix->dim * 4, (size_t)n,
                             on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
    launch_row_norms(X.p, ix->dpad, n, ix->dim, xn.p, xn2.p, st);
    assign_rows(*ix, X.p, ix->dpad, xn.p, xn2.p, n, a.p, st);
    M3G_CK(cudaMemcpyAsync(out, a.p, (size_t)n * 4,
                           on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
    M3G_CK(cudaStreamSynchronize(st));
}

// m3_async.cpp:262-313, clusters enqueued in ascending id order.
bool Engine::enqueue_insert_auto(int index_id, const int64_t* ids, const float* vecs, int64_t n) {
    auto ix = get(index_id, "AsyncEngine::enqueue_insert_auto");
    if (n == 0) return true;
    if (n < 0 || !ids || !vecs)
        fail(M3G_EINVAL, "AsyncEngine::enqueue_insert_auto: vecs size mismatch");
    std::vector<int32_t> assign((size_t)n);
    nearest_clusters(index_id, vecs, n, assign.data());
    for (int64_t i = 0; i < n; ++i)
        if (assign[(size_t)i] < 0)
            fail(M3G_ERUNTIME, "AsyncEngine::enqueue_insert_auto: unable to assign cluster");
    // one op carrying every row and its list: the writer applies it as one
    // add_batch per list (ascending list id, rows in call order), under one lock
    // with one staging copy and one scatter, instead of one queued op per list
    WriteOp op;
    op.kind = WriteOp::kInsertRouted;
    op.index_id = index_id;
    op.cluster_id = -1;
    op.ids.assign(ids, ids + n);
    op.vecs.assign(vecs, vecs + n * (int64_t)ix->dim);
    op.clusters = std::move(assign);
    return enqueue(std::move(op));
}

// ---------------- k-means / split ----------------

namespace {
// Device k-means over n rows of X (device, stride ld, zero padded to dpad).
// C (device, [nlist, dpad]) holds the start centroids and returns the result.
void kmeans_device(const float* X, int64_t ld, int64_t n, int dim, int dpad, int metric,
                   bool normalized, int nlist, int niter, float* C, int32_t* assign,
                   cudaStream_t st, int num_sms) {
    (void)num_sms;
    DBuf<float> xn, xn2, cn, cn2, S;
    xn.alloc((size_t)n);
    xn2.alloc((size_t)n);
    cn.alloc((size_t)nlist);
    cn2.alloc((size_t)nlist);
    launch_row_norms(X, ld, n, dim, xn.p, xn2.p, st);
    const int64_t ch = std::max<int64_t>(
        1, std::min<int64_t>({n, kMaxScoreEntries / std::max(nlist, 1), kMaxAssignRows}));
    S.alloc((size_t)(ch * nlist));
    const int64_t chunk = sort_chunk_rows(n, nlist);
    const int64_t nchunks = (n + chunk - 1) / chunk;
    DBuf<int32_t> counts, totals;
    DBuf<int64_t> start, perm;
    DBuf<__nv_bfloat16> X3, C3;
    DBuf<int> err;
    err.alloc(1);
    M3G_CK(cudaMemsetAsync(err.p, 0, sizeof(int), st));
    const int kp = gemm_tc_kdim(dpad);
    if (use_tc_gemm()) {
        X3.alloc((size_t)(ch * kp));
        C3.alloc((size_t)nlist * kp);
    }
    counts.alloc((size_t)(nchunks * nlist));
    totals.alloc((size_t)nlist);
    start.alloc((size_t)nlist + 1);
    perm.alloc((size_t)n);
    const float gam = (float)(dim + 4) * 5.9604645e-8f * 1.01f;
    auto assign_all = [&]() {
        launch_row_norms(C, dpad, nlist, dim, cn.p, cn2.p, st);
        if (use_tc_gemm()) M3G_CK(launch_split3(C, dpad, nlist, dpad, kp, C3.p, true, st));
        for (int64_t r0 = 0; r0 < n; r0 += ch) {
            const int64_t m = std::min(ch, n - r0);
            if (use_tc_gemm())
                M3G_CK(launch_split3(X + r0 * ld, ld, m, dpad, kp, X3.p, false, st));
            const float beta = coarse_gemm(X + r0 * ld, ld, X3.p, C, dpad, C3.p, S.p, nlist,
                                           (int)m, nlist, dpad, err.p, st);
            M3G_CK(launch_select_probes(S.p, nlist, X + r0 * ld, ld, C, dpad, xn.p + r0, xn2.p + r0,
                                        cn.p, cn2.p, (int)m, nlist, dim, metric, normalized ? 1 : 0,
                                        beta, gam, 1, 1, assign + r0, st));
        }
    };
    for (int it = 0; it < niter; ++it) {
        assign_all();
        M3G_CK(launch_stable_cluster_sort(assign, n, nlist, chunk, counts.p, totals.p, start.p,
                                          perm.p, st));
        M3G_CK(launch_centroid_update(X, ld, perm.p, start.p, nlist, dim, C, dpad, st));
    }
    assign_all();
    M3G_CK(cudaStreamSynchronize(st));
    int herr = 0;
    M3G_CK(cudaMemcpy(&herr, err.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) fail(M3G_ETIMEOUT, "k-means: a device-side wait gave up");
}
}  // namespace

void Engine::kmeans(const float* X, int64_t n, int dim, int metric, bool normalized, int nlist,
                    int niter, uint64_t seed, float* C_out, int32_t* assign_out) {
    if (dim <= 0) fail(M3G_EINVAL, "kmeans: dim must be > 0");
    if (nlist <= 0 || nlist > n) fail(M3G_EINVAL, "kmeans: nlist must be in [1, n]");
    if (niter < 0) fail(M3G_EINVAL, "kmeans: niter < 0");
    if (!X || !C_out) fail(M3G_EINVAL, "kmeans: buffers missing");
    DeviceGuard g(device_);
    const int dpad = round_up4(dim);
    cudaStream_t st;
    M3G_CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    struct StreamGuard {
        cudaStream_t s;
        ~StreamGuard() { cudaStreamDestroy(s); }
    } sg{st};
    DBuf<float> dX, dC;
    DBuf<int32_t> da;
    dX.alloc((size_t)(n * dpad));
    dC.alloc((size_t)nlist * dpad);
    da.alloc((size_t)n);
    if (dpad != dim) M3G_CK(cudaMemsetAsync(dX.p, 0, (size_t)(n * dpad) * 4, st));
    h2d_rows(dX.p, dpad, X, dim, n, st);
    std::vector<int64_t> init((size_t)nlist);
    sample_rows(seed, n, nlist, init.data());
    DevIdx di;
    di.upload(init, st);
    M3G_CK(launch_gather_rows(dX.p, dpad, di.d.p, nlist, dpad, dC.p, dpad, st));
    kmeans_device(dX.p, dpad, n, dim, dpad, metric, normalized, nlist, niter, dC.p, da.p, st, num_sms_);
    M3G_CK(cudaMemcpy2DAsync(C_out, (size_t)dim * 4, dC.p, (size_t)dpad * 4, (size_t)dim * 4,
                             (size_t)nlist, cudaMemcpyDeviceToHost, st));
    if (assign_out)
        M3G_CK(cudaMemcpyAsync(assign_out, da.p, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    M3G_CK(cudaStreamSynchronize(st));
}

void Engine::train_ivf(int index_id, int dim, int metric, bool normalized, const int64_t* ids,
                       const float* X, int64_t n, int nlist, int niter, uint64_t seed,
                       float* C_out) {
    if (!ids) fail(M3G_EINVAL, "train_ivf: ids missing");
    std::vector<float> C((size_t)nlist * dim);
    std::vector<int32_t> a((size_t)n);
    kmeans(X, n, dim, metric, normalized, nlist, niter, seed, C.data(), a.data());
    create_ivf(index_id, dim, metric, normalized, C.data(), nlist);
    // stable grouping of rows by list, ascending row order
    std::vector<int64_t> cnt((size_t)nlist + 1, 0);
    for (int64_t i = 0; i < n; ++i) cnt[(size_t)a[(size_t)i] + 1]++;
    for (int l = 0; l < nlist; ++l) cnt[(size_t)l + 1] += cnt[(size_t)l];
    std::vector<int64_t> order((size_t)n);
    {
        std::vector<int64_t> cur(cnt.begin(), cnt.end() - 1);
        for (int64_t i = 0; i < n; ++i) order[(size_t)cur[(size_t)a[(size_t)i]]++] = i;
    }
    std::vector<int64_t> lid;
    std::vector<float> lv;
    for (int l = 0; l < nlist; ++l) {
        const int64_t b = cnt[(size_t)l], e = cnt[(size_t)l + 1];
        if (b == e) continue;
        lid.resize((size_t)(e - b));
        lv.resize((size_t)(e - b) * dim);
        for (int64_t i = b; i < e; ++i) {
            lid[(size_t)(i - b)] = ids[order[(size_t)i]];
            std::memcpy(&lv[(size_t)(i - b) * dim], X + order[(size_t)i] * dim, sizeof(float) * dim);
        }
        load_cluster(index_id, l, lid.data(), lv.data(), e - b);
    }
    if (C_out) std::copy(C.begin(), C.end(), C_out);
}

int Engine::split_cluster(int index_id, int cid, int niter, uint64_t seed) {
    auto ix = get(index_id, "split_cluster");
    if (niter < 0) fail(M3G_EINVAL, "split_cluster: niter < 0");
    DeviceGuard g(device_);
    std::unique_lock lk(ix->mu);
    if (cid < 0 || cid >= ix->nlist()) fail(M3G_ERANGE, "split_cluster: invalid cluster_id");
    if (ws_.done) M3G_CK(cudaEventSynchronize(ws_.done));
    list_compact(*ix, cid);
    ListMeta& L = ix->lists[cid];
    const int64_t n = L.len;
    if (n < 2) {
        refresh_list_meta(*ix);
        return -1;
    }
    cudaStream_t st = ix->wstream;
    const int dpad = ix->dpad;
    DBuf<float> dC, wide;
    DBuf<int32_t> da;
    dC.alloc((size_t)2 * dpad);
    da.alloc((size_t)n);
    // the list's rows as fp32 [n, dpad]: the arena itself, or bf16 rows widened
    const float* X = reinterpret_cast<const float*>(ix->row_ptr(L.off));
    if (ix->bf16_rows()) {
        wide.alloc((size_t)(n * dpad));
        M3G_CK(launch_unpack_bf16_rows(reinterpret_cast<const __nv_bfloat16*>(ix->row_ptr(L.off)),
                                       ix->ldr, n, ix->dim, wide.p, dpad, st));
        X = wide.p;
    }
    int64_t init[2];
    sample_rows(seed, n, 2, init);
    std::vector<int64_t> init_abs = {init[0], init[1]};
    DevIdx di;
    di.upload(init_abs, st);
    M3G_CK(launch_gather_rows(X, dpad, di.d.p, 2, dpad, dC.p, dpad, st));
    kmeans_device(X, dpad, n, ix->dim, dpad, ix->metric, ix->normalized, 2, niter, dC.p, da.p, st,
                  num_sms_);
    std::vector<float> c2((size_t)2 * ix->dim);
    M3G_CK(cudaMemcpy2DAsync(c2.data(), (size_t)ix->dim * 4, dC.p, (size_t)dpad * 4,
                             (size_t)ix->dim * 4, 2, cudaMemcpyDeviceToHost, st));
    std::vector<int32_t> a((size_t)n);
    M3G_CK(cudaMemcpyAsync(a.data(), da.p, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    M3G_CK(cudaStreamSynchronize(st));
    std::vector<int64_t> side0, side1;
    for (int64_t r = 0; r < n; ++r) (a[(size_t)r] == 1 ? side1 : side0).push_back(r);
    // set_centroid(cid, c0); add_cluster(c1)  (m3_index.cpp:133-163)
    std::copy(c2.begin(), c2.begin() + ix->dim, ix->centroids.begin() + (size_t)cid * ix->dim);
    upload_centroids(*ix, cid, 1);
    const int nid = ix->nlist();
    ensure_centroid_cap(*ix, (size_t)nid + 1);
    ix->centroids.insert(ix->centroids.end(), c2.begin() + ix->dim, c2.end());
    ix->lists.emplace_back();
    upload_centroids(*ix, nid, 1);
    // rows regrouped in list order: side 1 to the new list, side 0 stays
    regroup_rows(*ix, cid, side1, nid);
    regroup_rows(*ix, cid, side0, cid);
    refresh_list_meta(*ix);
    return nid;
}

}  // namespace m3g
