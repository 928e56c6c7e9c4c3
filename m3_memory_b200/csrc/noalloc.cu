// noalloc.cu -- the exact top-nprobe centroid selection for callers that cannot
// allocate GPU memory.
//
// Some callers own every byte of device memory themselves: a host process that
// runs under a fixed memory budget with a pre-reserved pool, an embedding runtime
// that forbids allocations after start-up, or code that must not synchronise the
// device (cudaMalloc / cudaFree can).  They can call m3g_select_probes_noalloc:
// it runs the same three kernels as the engine's selection (row norms, the SIMT
// approximate GEMM, the exact selection) but keeps their scratch -- the
// approximate score matrix and the norms -- in one file-scope device array of
// fixed size, and calls no allocating routine.
//
// The array is kNoallocScratchBytes (16 MiB) and exists on every GPU that loads
// the library, for the life of the process.  All calls share it: two calls whose
// kernels overlap on the GPU race on it.  Every byte a call reads is written by
// the same call first, so nothing is carried over between calls.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "engine.h"
#include "kernels.h"
#include "kernels_kmeans.h"

namespace m3g {
namespace {

constexpr size_t kNoallocScratchBytes = size_t(16) << 20;
constexpr size_t kNoallocScratchFloats = kNoallocScratchBytes / sizeof(float);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoallocScratchFloats];

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once per
// device.  In host code the array's name is only a stand-in for the symbol.
float* noalloc_scratch(int dev) {
    if (dev < 0 || dev >= kMaxDevices) fail(M3G_EUNSUPPORTED, "select_probes_noalloc: device index too large");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();
            fail(M3G_ECUDA, std::string("select_probes_noalloc: cudaGetSymbolAddress: ") +
                                cudaGetErrorString(e));
        }
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    return g_noalloc_ptr[dev];
}

size_t align64(size_t n) { return (n + 63) & ~size_t(63); }

}  // namespace

// Scratch floats a call with these sizes needs.
size_t noalloc_scratch_floats(int64_t nq, int64_t nlist) {
    return align64((size_t)(nq * nlist)) + 2 * align64((size_t)nq) + 2 * align64((size_t)nlist);
}

void select_probes_noalloc(const float* dQ, int64_t nq, const float* dC, int64_t nlist, int dim,
                           int metric, int normalized, int nprobe, int32_t* d_out,
                           cudaStream_t st) {
    if (nq < 0 || nlist < 0 || dim <= 0) fail(M3G_EINVAL, "select_probes_noalloc: bad sizes");
    if (metric < 0 || metric > 2) fail(M3G_EINVAL, "select_probes_noalloc: unknown metric");
    if (nq == 0 || nlist == 0) return;
    if (!dQ || !dC || !d_out) fail(M3G_EINVAL, "select_probes_noalloc: null pointer");
    if (dim % 4 != 0 || (reinterpret_cast<uintptr_t>(dQ) & 15u) ||
        (reinterpret_cast<uintptr_t>(dC) & 15u))
        fail(M3G_EINVAL,
             "select_probes_noalloc: dim must be a multiple of 4 and the query / centroid "
             "arrays 16-byte aligned");
    if (dim > select_max_dim()) fail(M3G_EUNSUPPORTED, "select_probes_noalloc: dim too large");
    if (nlist > INT32_MAX / 2 || nq > INT32_MAX / 2)
        fail(M3G_EUNSUPPORTED, "select_probes_noalloc: too many rows");
    const int L = (int)nlist;
    const int P = nprobe <= 0 ? L : (int)std::min<int64_t>(nprobe, nlist);
    if (P >= L) {  // every list, in id order (as the engine does)
        M3G_CK(launch_iota_rows(d_out, nq, P, st));
        if (!st) M3G_CK(cudaStreamSynchronize(st));
        return;
    }
    const size_t need = noalloc_scratch_floats(nq, nlist);
    if (need > kNoallocScratchFloats)
        fail(M3G_EUNSUPPORTED,
             "select_probes_noalloc: nq * nlist too large for the fixed 16 MiB scratch "
             "(needs nq*nlist + 2 nq + 2 nlist <= 4194304 floats); split the queries");
    int dev = 0;
    M3G_CK(cudaGetDevice(&dev));
    float* base = noalloc_scratch(dev);
    float* S = base;
    float* qn = S + align64((size_t)(nq * nlist));
    float* qn2 = qn + align64((size_t)nq);
    float* cn = qn2 + align64((size_t)nq);
    float* cn2 = cn + align64((size_t)nlist);
    launch_row_norms(dQ, dim, nq, dim, qn, qn2, st);
    launch_row_norms(dC, dim, nlist, dim, cn, cn2, st);
    M3G_CK(cudaGetLastError());
    launch_sgemm_nt(dQ, dim, dC, dim, S, L, (int)nq, L, dim, st);
    M3G_CK(cudaGetLastError());
    const float gamma = (float)(dim + 4) * 5.9604645e-8f * 1.01f;
    M3G_CK(launch_select_probes(S, L, dQ, dim, dC, dim, qn, qn2, cn, cn2, (int)nq, L, dim, metric,
                                normalized, sgemm_error_beta(dim), gamma, P, 0, d_out, st));
    if (!st) M3G_CK(cudaStreamSynchronize(st));
}

}  // namespace m3g
