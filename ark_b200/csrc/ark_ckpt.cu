// ark_ckpt.cu -- ARK4 checkpoints written and read straight from ZeRO-1
// device shards (host code; no kernels).
//
// File format (proyecto_ark/ark01/src/io.rs:12-24, save_fp16 :432-500):
//   u32 magic "ARK4", u64 global_step, u64 adam_step, u64 n_tensors,
//   then per tensor: u64 n_elements, u64 type (0 = F16, 1 = F32), data;
//   tensor order: embed w (F16), m, v (F32); per layer the 9 weights
//   (wq wk wv wo w1 w2 w3 g1 g2, F16), their 9 m, their 9 v; gamma_final w,
//   m, v (training.rs:536-604).
// Appended after the last tensor (the reference's reader stops there and
// ignores it): u32 "ARKS", u32 64, then the 64-byte ark_opt_status, so the
// loss-scale state survives a restart (the reference restarts at 256,
// training.rs:120).
//
// Every rank of a sharded optimizer writes only the byte ranges of its own
// shard, with pwrite at offsets computed from the layout; rank 0 also sizes
// the file and writes the headers and the trailer.  Ranks need no barrier
// between them, but a reader must wait until every rank has returned.
// Reading is the mirror image (pread of the shard's ranges).  V3 files
// (FP32 weights and moments, no type field, io.rs:597-636) are read too;
// their weights are rounded to FP16 as memory.rs:347-377 does on resume.
#include <cuda_runtime.h>
#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>

#include <vector>

#include <cuda_fp16.h>

#include "ark_internal.h"

using namespace ark;

namespace {

constexpr uint32_t kMagicV4 = 0x4B345241u;   // "ARK4" little-endian
constexpr uint32_t kMagicV3 = 0x4B335241u;   // "ARK3"
constexpr uint32_t kMagicTrailer = 0x534B5241u;  // "ARKS"
constexpr size_t kHeaderV4 = 4 + 8 + 8 + 8;
constexpr size_t kStage = (size_t)64 << 20;  // pinned staging chunk

struct Record {
    uint32_t tensor;    // index into the model tensor list
    int kind;           // 0 = w (F16), 1 = m (F32), 2 = v (F32)
};

// File order of the 3 x T records for T = 2 + 9 L model tensors given in the
// order embed, l0.wq .. l0.g2, l1.wq .., gamma_final.
bool record_order(uint32_t T, std::vector<Record>& out) {
    if (T < 2 || (T - 2) % 9 != 0) return false;
    const uint32_t L = (T - 2) / 9;
    out.clear();
    for (int k = 0; k < 3; ++k) out.push_back({0u, k});
    for (uint32_t l = 0; l < L; ++l)
        for (int k = 0; k < 3; ++k)
            for (uint32_t i = 0; i < 9; ++i) out.push_back({1u + 9u * l + i, k});
    for (int k = 0; k < 3; ++k) out.push_back({T - 1, k});
    return true;
}

size_t elem_bytes(int kind) { return kind == 0 ? 2 : 4; }

bool write_all(int fd, const void* buf, size_t n, off_t off) {
    const char* p = static_cast<const char*>(buf);
    while (n) {
        const ssize_t w = pwrite(fd, p, n, off);
        if (w < 0 && errno == EINTR) continue;
        if (w <= 0) return false;
        p += w;
        n -= (size_t)w;
        off += w;
    }
    return true;
}

bool read_all(int fd, void* buf, size_t n, off_t off) {
    char* p = static_cast<char*>(buf);
    while (n) {
        const ssize_t r = pread(fd, p, n, off);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        p += r;
        n -= (size_t)r;
        off += r;
    }
    return true;
}

struct Pinned {
    void* p = nullptr;
    ~Pinned() {
        if (p) cudaFreeHost(p);
    }
};

// For each record: where its data starts in the file, given the layout.
void data_offsets(const ark_ckpt_tensor* t, const std::vector<Record>& recs, size_t header,
                  bool typed, std::vector<size_t>& off, size_t* end) {
    off.resize(recs.size());
    size_t o = header;
    for (size_t i = 0; i < recs.size(); ++i) {
        o += typed ? 16 : 8;
        off[i] = o;
        o += t[recs[i].tensor].numel * (typed ? elem_bytes(recs[i].kind) : 4);
    }
    *end = o;
}

// Intersection of a model tensor with this rank's shard [lo, lo+n).
bool shard_part(const ark_ckpt_tensor& t, uint64_t lo, uint64_t n, uint64_t* a, uint64_t* b) {
    const uint64_t s = t.flat_offset > lo ? t.flat_offset : lo;
    const uint64_t e0 = t.flat_offset + t.numel, e1 = lo + n;
    const uint64_t e = e0 < e1 ? e0 : e1;
    if (s >= e) return false;
    *a = s;
    *b = e;
    return true;
}

}  // namespace

extern "C" {

int ark_cuda_ckpt_save(ark_opt_state* st, const char* path, const ark_ckpt_tensor* tensors,
                       uint32_t n_tensors, uint64_t global_step, const uint16_t* w16,
                       const float* m, const float* v) {
    OptView c;
    if (!st || !path || !tensors || opt_view(st, &c)) return ARK_E_INVALID_ARG;
    std::vector<Record> recs;
    if (!record_order(n_tensors, recs)) return ARK_E_INVALID_ARG;
    if (c.n && (!w16 || !m || !v)) return ARK_E_INVALID_ARG;
    ark_opt_status status;
    int rc = ark_cuda_opt_read_status(st, &status);
    if (rc != ARK_OK && rc != ARK_E_EARLY_STOP) return rc;
    std::vector<size_t> off;
    size_t end = 0;
    data_offsets(tensors, recs, kHeaderV4, true, off, &end);
    const int fd = open(path, O_WRONLY | O_CREAT, 0644);
    if (fd < 0) return ARK_E_INVALID_ARG;
    bool ok = true;
    if (c.rank == 0) {
        // headers, record headers and trailer; the file gets its exact size
        ok = ftruncate(fd, (off_t)(end + 8 + sizeof(ark_opt_status))) == 0;
        char h[kHeaderV4];
        const uint64_t adam = status.opt_step, nt = recs.size();
        memcpy(h, &kMagicV4, 4);
        memcpy(h + 4, &global_step, 8);
        memcpy(h + 12, &adam, 8);
        memcpy(h + 20, &nt, 8);
        ok = ok && write_all(fd, h, sizeof(h), 0);
        for (size_t i = 0; i < recs.size() && ok; ++i) {
            const uint64_t rh[2] = {tensors[recs[i].tensor].numel,
                                    recs[i].kind == 0 ? 0ull : 1ull};
            ok = write_all(fd, rh, 16, (off_t)(off[i] - 16));
        }
        const uint32_t tr[2] = {kMagicTrailer, (uint32_t)sizeof(ark_opt_status)};
        ok = ok && write_all(fd, tr, 8, (off_t)end) &&
             write_all(fd, &status, sizeof(status), (off_t)(end + 8));
    }
    Pinned stage;
    if (ok && cudaMallocHost(&stage.p, kStage) != cudaSuccess) ok = false;
    int dev_prev = -1;
    cudaGetDevice(&dev_prev);
    cudaSetDevice(c.device);
    for (size_t i = 0; i < recs.size() && ok; ++i) {
        uint64_t a, b;
        if (!shard_part(tensors[recs[i].tensor], c.shard_offset, c.n, &a, &b)) continue;
        const size_t es = elem_bytes(recs[i].kind);
        const char* src = recs[i].kind == 0 ? reinterpret_cast<const char*>(w16)
                          : recs[i].kind == 1 ? reinterpret_cast<const char*>(m)
                                              : reinterpret_cast<const char*>(v);
        for (uint64_t x = a; x < b && ok;) {
            const uint64_t cnt = (b - x) * es < kStage ? (b - x) : kStage / es;
            ok = cudaMemcpy(stage.p, src + (x - c.shard_offset) * es, cnt * es,
                            cudaMemcpyDeviceToHost) == cudaSuccess &&
                 write_all(fd, stage.p, cnt * es,
                           (off_t)(off[i] + (x - tensors[recs[i].tensor].flat_offset) * es));
            x += cnt;
        }
    }
    if (dev_prev >= 0) cudaSetDevice(dev_prev);
    ok = (fsync(fd) == 0) && ok;
    close(fd);
    return ok ? ARK_OK : ARK_E_CUDA;
}

int ark_cuda_ckpt_load(ark_opt_state* st, const char* path, const ark_ckpt_tensor* tensors,
                       uint32_t n_tensors, uint64_t* global_step, uint16_t* w16, float* m,
                       float* v, uint32_t flags) {
    OptView c;
    if (!st || !path || !tensors || opt_view(st, &c)) return ARK_E_INVALID_ARG;
    if (flags & ~ARK_CKPT_RESTORE_SCALE) return ARK_E_INVALID_ARG;
    std::vector<Record> recs;
    if (!record_order(n_tensors, recs)) return ARK_E_INVALID_ARG;
    if (c.n && (!w16 || !m || !v)) return ARK_E_INVALID_ARG;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return ARK_E_INVALID_ARG;
    uint32_t magic = 0;
    uint64_t gstep = 0, adam = 0, nt = 0;
    bool ok = read_all(fd, &magic, 4, 0) && read_all(fd, &gstep, 8, 4);
    const bool v4 = magic == kMagicV4, v3 = magic == kMagicV3;
    ok = ok && (v4 || v3) && read_all(fd, &adam, 8, 12) && read_all(fd, &nt, 8, 20);
    // V3 files hold no gamma_final record (io.rs:608-620): 3 + 27 L records
    std::vector<Record> use = recs;
    if (ok && v3) {
        if (nt + 3 != recs.size()) ok = false;
        else use.erase(use.end() - 3, use.end());
    } else if (ok && nt != recs.size()) {
        ok = false;
    }
    std::vector<size_t> off;
    size_t end = 0;
    if (ok) data_offsets(tensors, use, kHeaderV4, v4, off, &end);
    // every record header must match the layout (no silent cold start)
    for (size_t i = 0; i < use.size() && ok; ++i) {
        uint64_t rh[2] = {0, 0};
        ok = read_all(fd, rh, v4 ? 16 : 8, (off_t)(off[i] - (v4 ? 16 : 8))) &&
             rh[0] == tensors[use[i].tensor].numel &&
             (!v4 || rh[1] == (use[i].kind == 0 ? 0ull : 1ull));
    }
    if (!ok) {
        close(fd);
        return ARK_E_INVALID_ARG;
    }
    Pinned stage;
    if (cudaMallocHost(&stage.p, kStage) != cudaSuccess) {
        close(fd);
        return ARK_E_CUDA;
    }
    int dev_prev = -1;
    cudaGetDevice(&dev_prev);
    cudaSetDevice(c.device);
    std::vector<uint16_t> tmp16;
    for (size_t i = 0; i < use.size() && ok; ++i) {
        uint64_t a, b;
        if (!shard_part(tensors[use[i].tensor], c.shard_offset, c.n, &a, &b)) continue;
        const int kind = use[i].kind;
        const size_t fes = v4 ? elem_bytes(kind) : 4, des = elem_bytes(kind);
        char* dst = kind == 0 ? reinterpret_cast<char*>(w16)
                    : kind == 1 ? reinterpret_cast<char*>(m)
                                : reinterpret_cast<char*>(v);
        for (uint64_t x = a; x < b && ok;) {
            const uint64_t cnt = (b - x) * fes < kStage ? (b - x) : kStage / fes;
            ok = read_all(fd, stage.p, cnt * fes,
                          (off_t)(off[i] + (x - tensors[use[i].tensor].flat_offset) * fes));
            const void* hsrc = stage.p;
            if (ok && kind == 0 && !v4) {   // V3 FP32 weights -> FP16, round to nearest even
                tmp16.resize(cnt);
                const float* f = static_cast<const float*>(stage.p);
                for (uint64_t j = 0; j < cnt; ++j) tmp16[j] = __half_as_ushort(__float2half_rn(f[j]));
                hsrc = tmp16.data();
            }
            ok = ok && cudaMemcpy(dst + (x - c.shard_offset) * des, hsrc, cnt * des,
                                  cudaMemcpyHostToDevice) == cudaSuccess;
            x += cnt;
        }
    }
    if (dev_prev >= 0) cudaSetDevice(dev_prev);
    // device state: the restored step (optimizer.rs:308); the loss scale as
    // saved in the trailer when asked for, else reset as the reference does
    ark_opt_status s;
    int rc = ok ? ark_cuda_opt_read_status(st, &s) : ARK_E_INVALID_ARG;
    if (rc == ARK_E_EARLY_STOP) rc = ARK_OK;
    if (rc == ARK_OK) {
        ark_opt_status saved;
        uint32_t tr[2] = {0, 0};
        const bool have = v4 && read_all(fd, tr, 8, (off_t)end) && tr[0] == kMagicTrailer &&
                          tr[1] == sizeof(saved) && read_all(fd, &saved, sizeof(saved), (off_t)(end + 8));
        ark_opt_status fresh;
        memset(&fresh, 0, sizeof(fresh));
        fresh.loss_scale = c.scale_init;
        fresh.last_clip_coef = 1.0f;
        if (have && (flags & ARK_CKPT_RESTORE_SCALE)) {
            fresh = saved;
            fresh.error = 0;
            fresh.steps_called = s.steps_called;   // epochs of the exchange continue
        } else {
            fresh.steps_called = s.steps_called;
        }
        fresh.opt_step = (uint32_t)adam;
        rc = ark_cuda_opt_set_status(st, &fresh);
    }
    close(fd);
    if (rc == ARK_OK && global_step) *global_step = gstep;
    return rc;
}

}  // extern "C"
