// faiss_io.cpp -- reads a Faiss IndexIVFFlat file straight into an engine
// index: the reference's only persistence path (rebuild_from_faiss,
// AgentMemory/M3/faiss_loader.py:24-79, which reads the file with the faiss
// package and calls create_ivf + load_cluster per list).  faiss is not needed
// here: the file is parsed from Faiss's published serialization layout
// (faiss/impl/index_write.cpp, format of IndexIVFFlat "IwFl" with an
// ArrayInvertedLists "ilar"):
//
//   u32 fourcc "IwFl"
//   index header: i32 d; i64 ntotal; i64 dummy x2; u8 is_trained; i32 metric
//                 (0 inner product, 1 L2); f32 metric_arg if metric > 1
//   u64 nlist; u64 nprobe
//   quantizer: u32 fourcc "IxF2" / "IxFI" / "IxFl" (IndexFlat), index header,
//              u64 n (floats), f32 centroids[n] (n = nlist * d)
//   direct map: u8 type; u64 n; i64[n]; (type 2: u64 m; (i64, i64)[m])
//   inverted lists: u32 fourcc "ilar"; u64 nlist; u64 code_size (d * 4);
//                   u32 "full": u64 n (= nlist); u64 sizes[n]
//                    or "sprs": u64 n (even); (u64 list, u64 size)[n / 2];
//                   then per non-empty list: u8 codes[size * code_size] (the
//                   fp32 vectors), i64 ids[size]
//                   (or u32 "il00": no lists)
//
// Only that plain form is read (the reference also accepts IVF indexes wrapped
// in other Faiss indexes via extract_index_ivf); anything else is refused with
// M3G_EUNSUPPORTED.  The metric maps as the reference maps it (L2 -> L2, inner
// product -> IP).  The whole file is read and checked before the index is
// replaced.
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "engine.h"

namespace m3g {
namespace {

struct Reader {
    FILE* f;
    std::string path;
    void bytes(void* p, size_t n) {
        if (n && std::fread(p, 1, n, f) != n)
            fail(M3G_ERUNTIME, "rebuild_from_faiss: truncated file: " + path);
    }
    template <class T>
    T one() {
        T v{};
        bytes(&v, sizeof(T));
        return v;
    }
    bool tag(const char* want) {
        char t[4];
        bytes(t, 4);
        return std::memcmp(t, want, 4) == 0;
    }
    void skip(uint64_t n) {
        if (n == 0) return;
        if (std::fseek(f, (long)n, SEEK_CUR) != 0)
            fail(M3G_ERUNTIME, "rebuild_from_faiss: truncated file: " + path);
    }
};

constexpr uint64_t kSane = uint64_t(1) << 40;

// i32 d; i64 ntotal; i64 x2; u8 is_trained; i32 metric (+ f32 arg)
void index_header(Reader& r, int* d, int64_t* ntotal, int* metric) {
    *d = r.one<int32_t>();
    *ntotal = r.one<int64_t>();
    r.one<int64_t>();
    r.one<int64_t>();
    r.one<uint8_t>();
    *metric = r.one<int32_t>();
    if (*metric > 1) r.one<float>();
    if (*d <= 0 || *ntotal < 0)
        fail(M3G_EINVAL, "rebuild_from_faiss: bad index header in " + r.path);
}

}  // namespace

void Engine::rebuild_from_faiss(int index_id, const char* path, bool normalized, int storage) {
    if (!path) fail(M3G_EINVAL, "rebuild_from_faiss: path missing");
    FILE* fp = std::fopen(path, "rb");
    if (!fp) fail(M3G_ERUNTIME, std::string("Faiss index file not found: ") + path);
    std::unique_ptr<FILE, int (*)(FILE*)> guard(fp, std::fclose);
    Reader r{fp, path};
    char top[4];
    r.bytes(top, 4);
    if (std::memcmp(top, "IwFl", 4) != 0)
        fail(M3G_EUNSUPPORTED, "rebuild_from_faiss: only a plain IndexIVFFlat file ('IwFl') is "
                               "read; found '" + std::string(top, 4) + "'");
    int d = 0, fmetric = 0;
    int64_t ntotal = 0;
    index_header(r, &d, &ntotal, &fmetric);
    int metric;
    if (fmetric == 1) metric = M3G_L2;
    else if (fmetric == 0) metric = M3G_IP;
    else fail(M3G_EINVAL, "Unsupported Faiss metric type: " + std::to_string(fmetric));
    const uint64_t nlist = r.one<uint64_t>();
    r.one<uint64_t>();  // nprobe
    if (nlist > (uint64_t)INT32_MAX / 2) fail(M3G_EINVAL, "rebuild_from_faiss: bad nlist");

    // quantizer: a flat index holding the nlist centroids
    char qt[4];
    r.bytes(qt, 4);
    if (std::memcmp(qt, "IxF2", 4) != 0 && std::memcmp(qt, "IxFI", 4) != 0 &&
        std::memcmp(qt, "IxFl", 4) != 0)
        fail(M3G_EUNSUPPORTED, "rebuild_from_faiss: the quantizer is not a flat index ('" +
                                   std::string(qt, 4) + "')");
    int qd = 0, qm = 0;
    int64_t qn = 0;
    index_header(r, &qd, &qn, &qm);
    const uint64_t nflt = r.one<uint64_t>();
    if (qd != d || (uint64_t)qn != nlist || nflt != nlist * (uint64_t)d)
        fail(M3G_EINVAL, "rebuild_from_faiss: quantizer does not hold nlist x d centroids");
    std::vector<float> C((size_t)nflt);
    r.bytes(C.data(), C.size() * 4);

    // direct map (ids -> list positions): not needed, skipped
    const uint8_t dm_type = r.one<uint8_t>();
    const uint64_t dm_n = r.one<uint64_t>();
    if (dm_n > kSane) fail(M3G_EINVAL, "rebuild_from_faiss: bad direct map");
    r.skip(dm_n * 8);
    if (dm_type == 2) {
        const uint64_t m = r.one<uint64_t>();
        if (m > kSane) fail(M3G_EINVAL, "rebuild_from_faiss: bad direct map");
        r.skip(m * 16);
    }

    // inverted lists
    std::vector<uint64_t> sizes((size_t)nlist, 0);
    std::vector<std::vector<int64_t>> ids((size_t)nlist);
    std::vector<std::vector<float>> vecs((size_t)nlist);
    char it[4];
    r.bytes(it, 4);
    if (std::memcmp(it, "ilar", 4) == 0) {
        const uint64_t ln = r.one<uint64_t>();
        const uint64_t code_size = r.one<uint64_t>();
        if (ln != nlist) fail(M3G_EINVAL, "rebuild_from_faiss: inverted lists disagree on nlist");
        if (code_size != (uint64_t)d * 4)
            fail(M3G_EUNSUPPORTED, "Only IndexIVFFlat (float codes) is supported for now");
        char lt[4];
        r.bytes(lt, 4);
        const uint64_t n = r.one<uint64_t>();
        if (n > kSane) fail(M3G_EINVAL, "rebuild_from_faiss: bad list sizes");
        if (std::memcmp(lt, "full", 4) == 0) {
            if (n != nlist) fail(M3G_EINVAL, "rebuild_from_faiss: bad list sizes");
            r.bytes(sizes.data(), (size_t)n * 8);
        } else if (std::memcmp(lt, "sprs", 4) == 0) {
            if (n % 2) fail(M3G_EINVAL, "rebuild_from_faiss: bad sparse list sizes");
            std::vector<uint64_t> pairs((size_t)n);
            r.bytes(pairs.data(), (size_t)n * 8);
            for (uint64_t i = 0; i < n; i += 2) {
                if (pairs[(size_t)i] >= nlist) fail(M3G_EINVAL, "rebuild_from_faiss: bad list id");
                sizes[(size_t)pairs[(size_t)i]] = pairs[(size_t)i + 1];
            }
        } else {
            fail(M3G_EINVAL, "rebuild_from_faiss: unknown list size format");
        }
        uint64_t total = 0;
        for (uint64_t l = 0; l < nlist; ++l) {
            const uint64_t s = sizes[(size_t)l];
            total += s;
            if (s > kSane / (uint64_t)d || total > kSane)
                fail(M3G_EINVAL, "rebuild_from_faiss: bad list size");
            if (s == 0) continue;
            vecs[(size_t)l].resize((size_t)(s * d));
            ids[(size_t)l].resize((size_t)s);
            r.bytes(vecs[(size_t)l].data(), (size_t)(s * code_size));
            r.bytes(ids[(size_t)l].data(), (size_t)s * 8);
        }
    } else if (std::memcmp(it, "il00", 4) != 0) {
        fail(M3G_EUNSUPPORTED, "rebuild_from_faiss: inverted lists of type '" +
                                   std::string(it, 4) + "' are not read");
    }
    create_ivf(index_id, d, metric, normalized, C.data(), (int64_t)nlist, storage);
    for (uint64_t l = 0; l < nlist; ++l)
        if (!ids[(size_t)l].empty())
            load_cluster(index_id, (int)l, ids[(size_t)l].data(), vecs[(size_t)l].data(),
                         (int64_t)ids[(size_t)l].size());
}

}  // namespace m3g
