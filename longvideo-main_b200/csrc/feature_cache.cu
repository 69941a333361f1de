// feature_cache.cu -- reader for the per-video feature cache (host code).
//
// Format (README.md section 3.2 and data_pipeline/src/npz_to_npy.py of the
// reference): <vid>.npy holds the frame features, C-order, little-endian
// float16 or float32, shape (L, P, d) or (L, d); <vid>.ts.npy holds the L
// frame timestamps (float32 or float64).  The reference reads them with
// numpy.load(mmap_mode="r") (cst_ssm/data/dataset.py:58-67).  Here the
// feature file is mapped read-only and frames are copied out of the mapping
// in parallel (std::thread) -- into a caller buffer, or into a pinned staging
// buffer followed by an asynchronous copy to the device, so a caller can
// upload chunk k+1 while it computes on chunk k.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "eacs_host.h"
#include "../../include/eacs_b200.h"

struct eacs_fc {
    int fd = -1;
    const unsigned char* map = nullptr;
    size_t map_len = 0;
    size_t data_off = 0;
    int64_t L = 0, P = 1, d = 0;
    int dtype = EACS_DTYPE_F16;
    size_t esz = 2;
    std::vector<float> ts;
};

namespace eacs {
namespace {

// Parse a .npy header: magic, version, header length, then the dict
// {'descr': ..., 'fortran_order': ..., 'shape': (...), }.
int parse_npy(const unsigned char* p, size_t len, std::string* descr, bool* fortran,
              std::vector<int64_t>* shape, size_t* data_off, const char* what) {
    if (len < 10 || std::memcmp(p, "\x93NUMPY", 6) != 0)
        return fail(EACS_ERR_INVALID, "feature cache: %s is not a .npy file", what);
    const int major = p[6];
    size_t hlen, hoff;
    if (major == 1) {
        hlen = p[8] | (p[9] << 8);
        hoff = 10;
    } else if (major == 2 || major == 3) {
        if (len < 12) return fail(EACS_ERR_INVALID, "feature cache: %s: truncated header", what);
        hlen = static_cast<size_t>(p[8]) | (static_cast<size_t>(p[9]) << 8) |
               (static_cast<size_t>(p[10]) << 16) | (static_cast<size_t>(p[11]) << 24);
        hoff = 12;
    } else {
        return fail(EACS_ERR_UNSUPPORTED, "feature cache: %s: .npy version %d", what, major);
    }
    if (hoff + hlen > len) return fail(EACS_ERR_INVALID, "feature cache: %s: truncated header", what);
    const std::string h(reinterpret_cast<const char*>(p + hoff), hlen);
    auto value_after = [&](const char* key) -> size_t {
        const size_t k = h.find(key);
        if (k == std::string::npos) return std::string::npos;
        const size_t c = h.find(':', k);
        return c == std::string::npos ? c : c + 1;
    };
    size_t v = value_after("'descr'");
    if (v == std::string::npos) return fail(EACS_ERR_INVALID, "feature cache: %s: no descr", what);
    const size_t q0 = h.find('\'', v), q1 = q0 == std::string::npos ? q0 : h.find('\'', q0 + 1);
    if (q1 == std::string::npos) return fail(EACS_ERR_INVALID, "feature cache: %s: bad descr", what);
    *descr = h.substr(q0 + 1, q1 - q0 - 1);
    v = value_after("'fortran_order'");
    if (v == std::string::npos) return fail(EACS_ERR_INVALID, "feature cache: %s: no fortran_order", what);
    const size_t fv = h.find_first_not_of(' ', v);
    if (fv == std::string::npos) return fail(EACS_ERR_INVALID, "feature cache: %s: bad fortran_order", what);
    *fortran = h.compare(fv, 4, "True") == 0;
    v = value_after("'shape'");
    const size_t s0 = v == std::string::npos ? v : h.find('(', v);
    const size_t s1 = s0 == std::string::npos ? s0 : h.find(')', s0);
    if (s1 == std::string::npos) return fail(EACS_ERR_INVALID, "feature cache: %s: bad shape", what);
    shape->clear();
    const std::string dims = h.substr(s0 + 1, s1 - s0 - 1);
    size_t i = 0;
    while (i < dims.size()) {
        while (i < dims.size() && (dims[i] == ' ' || dims[i] == ',')) ++i;
        if (i >= dims.size()) break;
        char* end = nullptr;
        const long long x = std::strtoll(dims.c_str() + i, &end, 10);
        if (end == dims.c_str() + i || x < 0)
            return fail(EACS_ERR_INVALID, "feature cache: %s: bad shape", what);
        shape->push_back(x);
        i = static_cast<size_t>(end - dims.c_str());
    }
    *data_off = hoff + hlen;
    return EACS_OK;
}

int map_file(const char* path, int* fd, const unsigned char** map, size_t* len) {
    *fd = ::open(path, O_RDONLY);
    if (*fd < 0) return fail(EACS_ERR_INVALID, "feature cache: cannot open %s", path);
    struct stat st;
    if (fstat(*fd, &st) != 0 || st.st_size <= 0) {
        ::close(*fd);
        *fd = -1;
        return fail(EACS_ERR_INVALID, "feature cache: cannot stat %s", path);
    }
    *len = static_cast<size_t>(st.st_size);
    void* m = mmap(nullptr, *len, PROT_READ, MAP_SHARED, *fd, 0);
    if (m == MAP_FAILED) {
        ::close(*fd);
        *fd = -1;
        return fail(EACS_ERR_INVALID, "feature cache: cannot map %s", path);
    }
    *map = static_cast<const unsigned char*>(m);
    return EACS_OK;
}

// Copy `bytes` from the mapping with up to `threads` threads (page faults of
// a cold file are then serviced in parallel).
void par_copy(void* dst, const void* src, size_t bytes) {
    const size_t min_part = 8u << 20;
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t parts = std::min<size_t>(std::min<size_t>(hw, 16), std::max<size_t>(1, bytes / min_part));
    if (parts <= 1) {
        std::memcpy(dst, src, bytes);
        return;
    }
    std::vector<std::thread> th;
    const size_t step = (bytes + parts - 1) / parts;
    for (size_t i = 0; i < parts; ++i) {
        const size_t o = i * step;
        if (o >= bytes) break;
        const size_t n = std::min(step, bytes - o);
        th.emplace_back([=] {
            std::memcpy(static_cast<char*>(dst) + o, static_cast<const char*>(src) + o, n);
        });
    }
    for (auto& t : th) t.join();
}

}  // namespace
}  // namespace eacs

using eacs::fail;

extern "C" {

int eacs_fc_open(const char* path, eacs_fc** out) {
    if (!path || !out) return fail(EACS_ERR_INVALID, "eacs_fc_open: null argument");
    *out = nullptr;
    auto* fc = new eacs_fc();
    int rc = eacs::map_file(path, &fc->fd, &fc->map, &fc->map_len);
    if (rc) {
        delete fc;
        return rc;
    }
    std::string descr;
    bool fortran = false;
    std::vector<int64_t> shape;
    rc = eacs::parse_npy(fc->map, fc->map_len, &descr, &fortran, &shape, &fc->data_off, path);
    if (!rc && fortran) rc = fail(EACS_ERR_UNSUPPORTED, "feature cache: %s is Fortran-ordered", path);
    if (!rc && descr != "<f2" && descr != "<f4")
        rc = fail(EACS_ERR_UNSUPPORTED, "feature cache: %s has dtype %s (float16 or float32 expected)",
                  path, descr.c_str());
    if (!rc && (shape.size() < 2 || shape.size() > 3))
        rc = fail(EACS_ERR_INVALID, "feature cache: %s: shape must be (L, P, d) or (L, d)", path);
    if (!rc) {
        fc->L = shape[0];
        fc->P = shape.size() == 3 ? shape[1] : 1;
        fc->d = shape.back();
        fc->dtype = descr == "<f2" ? EACS_DTYPE_F16 : EACS_DTYPE_F32;
        fc->esz = descr == "<f2" ? 2 : 4;
        // element count and byte size with overflow checks: a crafted header
        // must not wrap the product past the truncation check
        size_t elems = 0, bytes = 0, need = 0;
        if (__builtin_mul_overflow(static_cast<size_t>(fc->L), static_cast<size_t>(fc->P), &elems) ||
            __builtin_mul_overflow(elems, static_cast<size_t>(fc->d), &elems) ||
            __builtin_mul_overflow(elems, static_cast<size_t>(fc->esz), &bytes) ||
            __builtin_add_overflow(bytes, static_cast<size_t>(fc->data_off), &need))
            rc = fail(EACS_ERR_INVALID, "feature cache: %s: shape too large", path);
        else if (need > fc->map_len)
            rc = fail(EACS_ERR_INVALID, "feature cache: %s is truncated", path);
    }
    // timestamps: <path minus .npy>.ts.npy
    if (!rc) {
        std::string ts_path(path);
        if (ts_path.size() > 4 && ts_path.compare(ts_path.size() - 4, 4, ".npy") == 0)
            ts_path.resize(ts_path.size() - 4);
        ts_path += ".ts.npy";
        int tfd = -1;
        const unsigned char* tmap = nullptr;
        size_t tlen = 0;
        rc = eacs::map_file(ts_path.c_str(), &tfd, &tmap, &tlen);
        if (!rc) {
            std::string td;
            bool tf = false;
            std::vector<int64_t> tshape;
            size_t toff = 0;
            rc = eacs::parse_npy(tmap, tlen, &td, &tf, &tshape, &toff, ts_path.c_str());
            if (!rc && (tshape.size() != 1 || tshape[0] != fc->L))
                rc = fail(EACS_ERR_INVALID, "feature cache: %s holds %lld timestamps for %lld frames",
                          ts_path.c_str(), tshape.empty() ? -1LL : (long long)tshape[0], (long long)fc->L);
            if (!rc && td != "<f4" && td != "<f8")
                rc = fail(EACS_ERR_UNSUPPORTED, "feature cache: %s has dtype %s", ts_path.c_str(), td.c_str());
            if (!rc && toff + static_cast<size_t>(fc->L) * (td == "<f4" ? 4 : 8) > tlen)
                rc = fail(EACS_ERR_INVALID, "feature cache: %s is truncated", ts_path.c_str());
            if (!rc) {
                fc->ts.resize(static_cast<size_t>(fc->L));
                for (int64_t l = 0; l < fc->L; ++l) {
                    if (td == "<f4") {
                        float v;
                        std::memcpy(&v, tmap + toff + 4 * l, 4);
                        fc->ts[l] = v;
                    } else {
                        double v;
                        std::memcpy(&v, tmap + toff + 8 * l, 8);
                        fc->ts[l] = static_cast<float>(v);
                    }
                }
            }
            munmap(const_cast<unsigned char*>(tmap), tlen);
            ::close(tfd);
        }
    }
    if (rc) {
        munmap(const_cast<unsigned char*>(fc->map), fc->map_len);
        ::close(fc->fd);
        delete fc;
        return rc;
    }
    *out = fc;
    return EACS_OK;
}

int eacs_fc_info(const eacs_fc* fc, int64_t* L, int64_t* P, int64_t* d, int* dtype) {
    if (!fc) return fail(EACS_ERR_INVALID, "eacs_fc_info: null handle");
    if (L) *L = fc->L;
    if (P) *P = fc->P;
    if (d) *d = fc->d;
    if (dtype) *dtype = fc->dtype;
    return EACS_OK;
}

int eacs_fc_timestamps(const eacs_fc* fc, float* out) {
    if (!fc || !out) return fail(EACS_ERR_INVALID, "eacs_fc_timestamps: null argument");
    std::memcpy(out, fc->ts.data(), sizeof(float) * fc->ts.size());
    return EACS_OK;
}

int eacs_fc_read(const eacs_fc* fc, int64_t l0, int64_t n, void* dst) {
    if (!fc || (!dst && n > 0)) return fail(EACS_ERR_INVALID, "eacs_fc_read: null argument");
    if (l0 < 0 || n < 0 || l0 + n > fc->L)
        return fail(EACS_ERR_INVALID, "eacs_fc_read: frames [%lld, %lld) outside [0, %lld)", (long long)l0,
                    (long long)(l0 + n), (long long)fc->L);
    const size_t frame = static_cast<size_t>(fc->P * fc->d) * fc->esz;
    eacs::par_copy(dst, fc->map + fc->data_off + static_cast<size_t>(l0) * frame, static_cast<size_t>(n) * frame);
    return EACS_OK;
}

int eacs_fc_upload(const eacs_fc* fc, int64_t l0, int64_t n, void* staging, size_t staging_bytes,
                   void* dst_device, void* stream) {
    if (!fc || !staging || !dst_device) return fail(EACS_ERR_INVALID, "eacs_fc_upload: null argument");
    const size_t bytes = static_cast<size_t>(n) * static_cast<size_t>(fc->P * fc->d) * fc->esz;
    if (staging_bytes < bytes)
        return fail(EACS_ERR_WORKSPACE, "eacs_fc_upload: staging of %zu bytes needed, %zu given", bytes,
                    staging_bytes);
    int rc = eacs_fc_read(fc, l0, n, staging);
    if (rc) return rc;
    return eacs::cuda_check(cudaMemcpyAsync(dst_device, staging, bytes, cudaMemcpyHostToDevice,
                                            static_cast<cudaStream_t>(stream)),
                            "eacs_fc_upload");
}

void eacs_fc_close(eacs_fc* fc) {
    if (!fc) return;
    if (fc->map) munmap(const_cast<unsigned char*>(fc->map), fc->map_len);
    if (fc->fd >= 0) ::close(fc->fd);
    delete fc;
}

}  // extern "C"
