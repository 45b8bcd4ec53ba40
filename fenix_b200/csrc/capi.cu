// capi.cu — the extern "C" boundary (include/fenix_b200.h). Statuses map 1:1 to the
// reference's fenix::Errc; no exception crosses the ABI; messages go to a thread-local
// last-error string.
#include "fenix_b200.h"
#include "fenix_b200/ml/tiling.hpp"
#include "net.cuh"
#include "counters.hpp"
#include "pack.cuh"
#include "ptx.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

namespace fxh {
extern unsigned long long* g_conv_trace;
}


// Static device scratch of fx_norm_tiles_noalloc: the tile origins, then the per-tile exact
// sums (Σv, Σv² as u64). One copy per device (a __device__ variable lives in every context).
// Concurrent calls on one device share it and race.
namespace {
constexpr int kNoAllocMaxTiles = 4096;
constexpr size_t kNoAllocOrgBytes = sizeof(fxk::TileOrigin) * kNoAllocMaxTiles;        // 96 KiB
constexpr size_t kNoAllocSumBytes = 2 * sizeof(unsigned long long) * kNoAllocMaxTiles;  // 64 KiB
static_assert(kNoAllocOrgBytes % 256 == 0, "sums must start 256-byte aligned");
static_assert(sizeof(fxk::TileOrigin) == 3 * sizeof(int64_t), "origins are copied as int64 triples");
constexpr int kNoAllocMaxDevices = 64;
}  // namespace
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocOrgBytes + kNoAllocSumBytes];

namespace {

thread_local std::string g_last_error;

fx_status set_err(const fxh::Status& st) {
    g_last_error = st.msg;
    return static_cast<fx_status>(st.code);
}
fx_status set_err(int code, const std::string& m) {
    g_last_error = m;
    return static_cast<fx_status>(code);
}

template <class F>
fx_status guarded(F&& f) {
    try {
        g_last_error.clear();
        return f();
    } catch (const std::bad_alloc&) {
        return set_err(FX_INTERNAL, "out of host memory");
    } catch (const std::exception& e) {
        return set_err(FX_INTERNAL, std::string("internal error: ") + e.what());
    } catch (...) {
        return set_err(FX_INTERNAL, "internal error");
    }
}

}  // namespace

namespace fxh {
fx_status abi_error(int code, const std::string& msg) { return set_err(code, msg); }
fx_status abi_exception() {
    try {
        throw;
    } catch (const std::bad_alloc&) {
        return set_err(FX_INTERNAL, "out of host memory");
    } catch (const std::exception& e) {
        return set_err(FX_INTERNAL, std::string("internal error: ") + e.what());
    } catch (...) {
        return set_err(FX_INTERNAL, "internal error");
    }
}
// The tile of a call: opts.tile when set (all three positive), else the cube of side opts.patch,
// which must be divisible by 64 as in the reference (src/ml/infer.hpp:459).
fx_status opts_tile(const fx_infer_opts* o, fxk::TileDims* t) {
    if (o->tile[0] == 0 && o->tile[1] == 0 && o->tile[2] == 0) {
        if (o->patch <= 0 || o->patch % 64 != 0) return set_err(FX_INVALID_ARGUMENT, "patch must be divisible by 64");
        *t = {o->patch, o->patch, o->patch};
        return FX_OK;
    }
    if (o->tile[0] <= 0 || o->tile[1] <= 0 || o->tile[2] <= 0)
        return set_err(FX_INVALID_ARGUMENT, "tile: all three extents must be positive");
    *t = {o->tile[0], o->tile[1], o->tile[2]};
    return FX_OK;
}

// ml::InferOptions fields beyond the tile grid, as the driver's per-call options.
RunOpts run_opts(const fx_infer_opts* o) {
    RunOpts r;
    r.norm = o->norm;
    r.skip_constant = o->skip_constant != 0;
    r.filter = o->tile_filter;
    r.filter_user = o->tile_filter_user;
    for (int a = 0; a < 3; ++a) {
        r.core_org[a] = o->core_org[a];
        r.core_ext[a] = o->core_ext[a];
    }
    r.stacks = std::max(o->stacks, 1);
    return r;
}

// The output crop of opts over an input of dims d (src/ml/infer.hpp:462-472): origin clamped into
// the input, extent (<= 0: to the end) clamped to it.
void crop_box(const fx_infer_opts* o, const int64_t d[3], int64_t co[3], int64_t ce[3]) {
    for (int a = 0; a < 3; ++a) {
        co[a] = std::clamp<int64_t>(o->core_org[a], 0, d[a]);
        ce[a] = o->core_ext[a] <= 0 ? d[a] - co[a] : std::min(o->core_ext[a], d[a] - co[a]);
    }
}

// ---- resumable prediction: the reference's FXICKPT3 checkpoint (src/ml/infer.hpp:136-344) ----
// The header is the reference's struct, field for field (the same bytes on disk, so either side
// resumes the other's file); the trailing 4 bytes of padding are zero.
struct CkptHeader {
    char magic[8] = {'F', 'X', 'I', 'C', 'K', 'P', 'T', '3'};
    int64_t dz = 0, dy = 0, dx = 0;
    int64_t tile_shift = 0;
    int64_t total_tiles = 0;
    int64_t n_done = 0;
    uint64_t weights_hash = 0, input_hash = 0;
    double overlap = 0, acc_scale = 0;
    int32_t patch = 0, tta = 0, channel = 0, sigmoid = 0, norm = 0;
};
static_assert(sizeof(CkptHeader) == 112, "FXICKPT3 header layout");

// Load a checkpoint that matches `want` into host f32 acc (nvox values): its completed tile count,
// or -1 (absent, mismatched, short or unreadable: acc untouched, start fresh).
int64_t ckpt_load(const std::string& path, const CkptHeader& want, std::vector<float>& acc) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return -1;
    CkptHeader h;
    const bool ok = std::fread(&h, sizeof h, 1, f) == 1 && std::memcmp(h.magic, want.magic, 8) == 0 &&
                    h.dz == want.dz && h.dy == want.dy && h.dx == want.dx && h.patch == want.patch &&
                    h.overlap == want.overlap && h.tta == want.tta && h.tile_shift == want.tile_shift &&
                    h.total_tiles == want.total_tiles && h.weights_hash == want.weights_hash &&
                    h.input_hash == want.input_hash && h.channel == want.channel && h.sigmoid == want.sigmoid &&
                    h.norm == want.norm && h.n_done >= 0 && h.n_done <= h.total_tiles;
    const size_t nvox = acc.size();
    int64_t n = -1;
    if (ok) {
        std::fseek(f, 0, SEEK_END);
        const long fsize = std::ftell(f);
        const long need = static_cast<long>(sizeof(CkptHeader) + (h.acc_scale > 0.0 ? nvox * sizeof(uint16_t) : 0));
        if (fsize >= need && std::fseek(f, sizeof(CkptHeader), SEEK_SET) == 0) {
            if (h.acc_scale <= 0.0) {
                std::fill(acc.begin(), acc.end(), 0.0f);
                n = h.n_done;
            } else {
                std::vector<uint16_t> q(nvox);
                if (std::fread(q.data(), sizeof(uint16_t), nvox, f) == nvox) {
                    const float sc = static_cast<float>(h.acc_scale / 65535.0);
                    for (size_t i = 0; i < nvox; ++i) acc[i] = static_cast<float>(q[i]) * sc;
                    n = h.n_done;
                }
            }
        }
    }
    std::fclose(f);
    return n;
}

// Header + u16 payload to path (temp + rename); best effort.
void ckpt_write(const std::string& path, const CkptHeader& h, const std::vector<uint16_t>& q) {
    const std::string tmp = path + ".tmp";
    std::FILE* f = std::fopen(tmp.c_str(), "wb");
    if (!f) return;
    bool ok = std::fwrite(&h, sizeof h, 1, f) == 1;
    if (ok && h.acc_scale > 0.0) ok = std::fwrite(q.data(), sizeof(uint16_t), q.size(), f) == q.size();
    ok = std::fflush(f) == 0 && ok;
    std::fclose(f);
    if (ok) std::rename(tmp.c_str(), path.c_str());
    else std::remove(tmp.c_str());
}

// The background writer: one write in flight; a save requested meanwhile is skipped.
struct CkptWriter {
    std::thread th;
    std::atomic<bool> busy{false};
    std::vector<uint16_t> q;
    ~CkptWriter() { join(); }
    void join() {
        if (th.joinable()) th.join();
    }
    // Snapshot d_acc (device max, quantise, D2H on stream s) and hand it to the writer thread.
    fx_status save(const std::string& path, CkptHeader h, const float* d_acc, size_t nvox, unsigned* d_max,
                   uint16_t* d_q, cudaStream_t s) {
        if (busy.load()) return FX_OK;
        join();
        unsigned bits = 0;
        cudaError_t e = cudaMemsetAsync(d_max, 0, sizeof(unsigned), s);
        if (e == cudaSuccess) e = fxk::launch_acc_max(d_acc, static_cast<int64_t>(nvox), d_max, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(&bits, d_max, sizeof bits, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return set_err(cuda_status(e, "checkpoint"));
        float mx;
        std::memcpy(&mx, &bits, sizeof mx);
        h.acc_scale = mx > 0.0f ? static_cast<double>(mx) : 0.0;
        if (h.acc_scale > 0.0) {
            q.resize(nvox);
            const float inv = static_cast<float>(65535.0 / h.acc_scale);
            e = fxk::launch_acc_quant_u16(d_acc, static_cast<int64_t>(nvox), inv, d_q, s);
            if (e == cudaSuccess) e = cudaMemcpyAsync(q.data(), d_q, nvox * sizeof(uint16_t), cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess) e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) return set_err(cuda_status(e, "checkpoint"));
        }
        busy = true;
        th = std::thread([this, path, h] {
            ckpt_write(path, h, q);
            busy = false;
        });
        return FX_OK;
    }
};

// predict_tiles over the whole grid with checkpointing: resume from a matching file, save every
// `every` tiles, remove the file on success (src/ml/infer.hpp:571-606, 790-861).
fx_status predict_ckpt(fx_net* n, const uint8_t* d_vol, int64_t dz, int64_t dy, int64_t dx, fxk::TileDims tl,
                       const fx_infer_opts* o, float* d_acc, cudaStream_t s) {
    if (tl.z != tl.y || tl.y != tl.x || std::max(o->stacks, 1) > 1 || o->tile_filter || o->skip_constant)
        return set_err(FX_UNSUPPORTED, "predict: checkpoints need a cubic tile, one volume, every tile (no filter)");
    const int64_t d[3] = {dz, dy, dx};
    int64_t co[3], ce[3];
    crop_box(o, d, co, ce);
    if (co[0] || co[1] || co[2] || ce[0] != dz || ce[1] != dy || ce[2] != dx)
        return set_err(FX_UNSUPPORTED, "predict: checkpoints take no output crop (src/ml/infer.hpp:575)");
    const std::string path(o->ckpt_path);
    const int64_t total = static_cast<int64_t>(fenix::ml::tile_starts(dz, tl.z, o->overlap).size() *
                                               fenix::ml::tile_starts(dy, tl.y, o->overlap).size() *
                                               fenix::ml::tile_starts(dx, tl.x, o->overlap).size());
    CkptHeader h;
    h.dz = dz;
    h.dy = dy;
    h.dx = dx;
    h.patch = tl.z;
    h.overlap = o->overlap;
    h.tta = o->tta;
    h.total_tiles = total;
    h.weights_hash = o->weights_hash;
    h.input_hash = o->input_hash;
    h.channel = o->channel;
    h.sigmoid = o->sigmoid ? 1 : 0;
    h.norm = o->norm;
    const size_t nvox = static_cast<size_t>(dz) * dy * dx;
    int64_t done = -1;
    {
        std::vector<float> host;
        if (std::FILE* f = std::fopen(path.c_str(), "rb")) {  // host copy only when there is a file
            std::fclose(f);
            host.resize(nvox);
            done = ckpt_load(path, h, host);
        }
        cudaError_t e = done >= 0 ? cudaMemcpyAsync(d_acc, host.data(), nvox * sizeof(float), cudaMemcpyHostToDevice, s)
                                  : cudaMemsetAsync(d_acc, 0, nvox * sizeof(float), s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return set_err(cuda_status(e, "checkpoint load"));
    }
    if (done < 0) done = 0;
    const int b = std::max(1, std::min(o->batch, n->net.max_batch()));
    int64_t every = o->ckpt_every > 0 ? o->ckpt_every : 128;
    every = (every + b - 1) / b * b;  // whole forwards between saves
    unsigned* d_max = nullptr;
    uint16_t* d_q = nullptr;
    if (cudaMalloc(&d_max, sizeof(unsigned)) != cudaSuccess || cudaMalloc(&d_q, nvox * sizeof(uint16_t)) != cudaSuccess) {
        cudaFree(d_max);
        return set_err(FX_INTERNAL, "cudaMalloc: checkpoint snapshot");
    }
    fx_status r = FX_OK;
    {
        CkptWriter w;
        for (int64_t t = done; t < total && r == FX_OK; t += every) {
            const int64_t t1 = std::min(total, t + every);
            Status st = n->net.predict_tiles(d_vol, dz, dy, dx, 0, dz, tl, o->overlap, o->channel, o->sigmoid, o->batch,
                                             t, t1, d_acc, s, 0, dz, o->tta, run_opts(o));
            if (!st.ok()) {
                r = set_err(st);
                break;
            }
            if (t1 < total) {
                h.n_done = t1;
                r = w.save(path, h, d_acc, nvox, d_max, d_q, s);
            }
        }
        w.join();
    }
    cudaFree(d_max);
    cudaFree(d_q);
    if (r == FX_OK) {
        std::remove(path.c_str());
        std::remove((path + ".tmp").c_str());
    }
    return r;
}

// The device part of fx_predict_volume (src/ml/infer.hpp:456-864 + inference.cpp:343-351): d_vol
// (resident, dims dz, dy, dx) -> Gaussian blend in d_acc (the crop's dims) -> normalised probability
// in d_prob (may alias d_acc) and/or u8 in d_u8. Runs on the net's stream and synchronises it.
fx_status predict_resident(fx_net* n, const uint8_t* d_vol, int64_t dz, int64_t dy, int64_t dx,
                           const fx_infer_opts* o, float* d_acc, float* d_prob, uint8_t* d_u8, cudaStream_t s,
                           bool sync) {
    if (!s) s = n->net.stream();
    const int64_t d[3] = {dz, dy, dx};
    int64_t co[3], ce[3];
    crop_box(o, d, co, ce);
    if (ce[0] < 1 || ce[1] < 1 || ce[2] < 1) return set_err(FX_INVALID_ARGUMENT, "predict: empty output crop");
    const int ns = std::max(o->stacks, 1);
    if (ns > 1 && (co[0] || co[1] || co[2] || ce[0] != dz || ce[1] != dy || ce[2] != dx))
        return set_err(FX_UNSUPPORTED, "predict: stacks take no output crop");
    const size_t nv = static_cast<size_t>(ce[0]) * ce[1] * ce[2];
    fxk::TileDims tl{};
    if (fx_status r = opts_tile(o, &tl)) return r;
    Status st = ok();
    if (o->ckpt_path && *o->ckpt_path) {
        if (fx_status r = predict_ckpt(n, d_vol, dz, dy, dx, tl, o, d_acc, s)) return r;
    } else {
        cudaMemsetAsync(d_acc, 0, nv * sizeof(float), s);
        st = n->net.predict_tiles(d_vol, dz, dy, dx, 0, dz, tl, o->overlap, o->channel, o->sigmoid, o->batch, 0, -1,
                                  d_acc, s, co[0], ce[0], o->tta, run_opts(o));
        if (!st.ok()) return set_err(st);
    }
    const int T[3] = {tl.z, tl.y, tl.x};
    std::vector<float> w(static_cast<size_t>(ce[0] + ce[1] + ce[2]));
    size_t at = 0;
    for (int a = 0; a < 3; ++a) {
        // the factorised weight over the crop's span of each axis (src/ml/infer.hpp:499-509); with
        // stacks, the z profile of one stack repeated
        const auto g = fenix::ml::gaussian1d(T[a]);
        const int64_t len = a == 0 ? d[0] / ns : d[a];
        const auto starts = fenix::ml::tile_starts(len, T[a], o->overlap);
        const auto W = fenix::ml::weight_profile(g, starts, a == 0 && ns > 1 ? 0 : co[a], a == 0 ? ce[0] / ns : ce[a],
                                                 len, T[a]);
        for (int k = 0; k < (a == 0 ? ns : 1); ++k) {
            std::copy(W.begin(), W.end(), w.begin() + static_cast<std::ptrdiff_t>(at));
            at += W.size();
        }
    }
    float* d_w = n->net.profile_buffer(w.size());
    if (!d_w) return set_err(FX_INTERNAL, "cudaMalloc: weight profiles");
    cudaMemcpyAsync(d_w, w.data(), sizeof(float) * w.size(), cudaMemcpyHostToDevice, s);
    cudaError_t e = fxk::launch_accum_finalize(d_acc, ce[0], ce[1], ce[2], 0, ce[0], d_w, d_w + ce[0],
                                               d_w + ce[0] + ce[1], d_prob, d_u8, s);
    if (e != cudaSuccess) return set_err(cuda_status(e, "accum_finalize"));
    if (sync) {
        if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return set_err(cuda_status(e, "predict"));
        if ((st = n->net.take_device_status()).code) return set_err(st);  // a bounded wait that gave up
    }
    return FX_OK;
}
}  // namespace fxh

namespace {

int sm_count_of_current() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

bool is_sm100() {
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    return major == 10;
}

// Scoped device allocations for the single-op entry points.
struct Scratch {
    std::vector<void*> ptrs;
    ~Scratch() {
        for (void* p : ptrs) cudaFree(p);
    }
    void* get(size_t bytes) {
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
        ptrs.push_back(p);
        return p;
    }
};

float device_absmax(const float* x, int64_t n, cudaStream_t s, Scratch& sc) {
    unsigned* d = static_cast<unsigned*>(sc.get(sizeof(unsigned)));
    if (!d) return 0.f;
    cudaMemsetAsync(d, 0, sizeof(unsigned), s);
    fxk::launch_absmax(x, n, d, s);
    unsigned bits = 0;
    cudaMemcpyAsync(&bits, d, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

}  // namespace

extern "C" {

const char* fx_last_error(void) { return g_last_error.c_str(); }

int fx_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

fx_status fx_net_create(const char* path, int patch, int max_batch, fx_precision precision, int device, fx_net** out) {
    return guarded([&]() -> fx_status {
        if (!path || !out) return set_err(FX_INVALID_ARGUMENT, "fx_net_create: null argument");
        *out = nullptr;
        auto h = std::make_unique<fx_net>();
        const int t[3] = {patch, patch, patch};
        fxh::Status st = h->net.create(path, t, max_batch, static_cast<int>(precision), device);
        if (!st.ok()) return set_err(st);
        *out = h.release();
        return FX_OK;
    });
}

fx_status fx_net_create_tiled(const char* path, const int tile[3], int max_batch, fx_precision precision, int device,
                              fx_net** out) {
    return guarded([&]() -> fx_status {
        if (!path || !tile || !out) return set_err(FX_INVALID_ARGUMENT, "fx_net_create_tiled: null argument");
        *out = nullptr;
        auto h = std::make_unique<fx_net>();
        fxh::Status st = h->net.create(path, tile, max_batch, static_cast<int>(precision), device);
        if (!st.ok()) return set_err(st);
        *out = h.release();
        return FX_OK;
    });
}

void fx_net_destroy(fx_net* net) { delete net; }

int fx_net_patch(const fx_net* n) { return n ? n->net.patch() : 0; }
int fx_net_tile(const fx_net* n, int tile[3], int* masks, int cap) {
    if (!n) return 0;
    const fxk::TileDims t = n->net.tile();
    if (tile) {
        tile[0] = t.z;
        tile[1] = t.y;
        tile[2] = t.x;
    }
    const auto& m = n->net.stage_masks();
    for (int i = 0; masks && i < cap && i < static_cast<int>(m.size()); ++i) masks[i] = m[i];
    return static_cast<int>(m.size());
}
int fx_net_max_batch(const fx_net* n) { return n ? n->net.max_batch() : 0; }
int fx_net_classes(const fx_net* n) { return n ? n->net.classes() : 0; }
int fx_net_features(const fx_net* n, int* out, int cap) {
    if (!n) return 0;
    const auto& f = n->net.features();
    for (int i = 0; i < cap && i < static_cast<int>(f.size()); ++i) out[i] = f[i];
    return static_cast<int>(f.size());
}

fx_status fx_net_calibrate(fx_net* n, const uint8_t* host_patches, int count) {
    return guarded([&]() -> fx_status {
        if (!n || !host_patches) return set_err(FX_INVALID_ARGUMENT, "fx_net_calibrate: null argument");
        fxh::Status st = n->net.calibrate(host_patches, count);
        return st.ok() ? FX_OK : set_err(st);
    });
}

fx_status fx_net_set_norm(fx_net* n, int norm) {
    if (!n || norm < FX_NORM_ZSCORE || norm > FX_NORM_UNIT255)
        return set_err(FX_INVALID_ARGUMENT, "fx_net_set_norm: bad argument");
    n->net.set_norm(norm);
    return FX_OK;
}

fx_status fx_net_set_act_scales(fx_net* n, const float* scales, int count) {
    return guarded([&]() -> fx_status {
        if (!n || !scales) return set_err(FX_INVALID_ARGUMENT, "fx_net_set_act_scales: null argument");
        fxh::Status st = n->net.set_act_scales(scales, count);
        return st.ok() ? FX_OK : set_err(st);
    });
}

fx_status fx_net_set_layer_precision(fx_net* n, const int* prec, int count) {
    return guarded([&]() -> fx_status {
        if (!n || !prec) return set_err(FX_INVALID_ARGUMENT, "fx_net_set_layer_precision: null argument");
        // fx_precision -> operand type: FX_PREC_FP8 = e4m3, FX_PREC_BF16 = bf16, FX_PREC_F16 = f16
        std::vector<int> q(static_cast<size_t>(std::max(count, 0)));
        for (int i = 0; i < count; ++i)
            q[i] = prec[i] == FX_PREC_FP8 ? fxk::kOpE4M3 : (prec[i] == FX_PREC_BF16 ? fxk::kOpBF16 : fxk::kOpF16);
        fxh::Status st = n->net.set_layer_precision(q.data(), count);
        return st.ok() ? FX_OK : set_err(st);
    });
}

fx_status fx_net_calibrate_schedule(fx_net* n, const uint8_t* host_patches, int count, double min_dice, double max_abs,
                                    double* dice, double* maxabs) {
    return guarded([&]() -> fx_status {
        if (!n || !host_patches) return set_err(FX_INVALID_ARGUMENT, "fx_net_calibrate_schedule: null argument");
        fxh::Status st = n->net.calibrate_schedule(host_patches, count, min_dice, max_abs, dice, maxabs);
        return st.ok() ? FX_OK : set_err(st);
    });
}

int fx_net_layer_precision(const fx_net* n, int* prec, double* flops, int cap) {
    if (!n) return 0;
    const auto q = n->net.layer_precision();
    const auto f = n->net.layer_flops();
    for (int i = 0; i < cap && i < static_cast<int>(q.size()); ++i) {
        if (prec) prec[i] = q[i] == fxk::kOpE4M3 ? FX_PREC_FP8 : (q[i] == fxk::kOpBF16 ? FX_PREC_BF16 : FX_PREC_F16);
        if (flops) flops[i] = f[i];
    }
    return static_cast<int>(q.size());
}

const char* fx_net_layer_name(const fx_net* n, int i) {
    const fxh::Layer* L = n ? n->net.layer_at(i) : nullptr;
    return L ? L->name.c_str() : nullptr;
}

int fx_net_act_scales(const fx_net* n, float* out, int cap) {
    if (!n) return 0;
    auto v = n->net.act_scales();
    for (int i = 0; i < cap && i < static_cast<int>(v.size()); ++i) out[i] = v[i];
    return static_cast<int>(v.size());
}

fx_status fx_net_forward(fx_net* n, const uint8_t* dev_tiles, int nb, float* dev_prob, int channel, int sigmoid,
                         void* stream) {
    return guarded([&]() -> fx_status {
        if (!n || !dev_tiles || !dev_prob) return set_err(FX_INVALID_ARGUMENT, "fx_net_forward: null argument");
        cudaSetDevice(n->net.device());
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : n->net.stream();
        const fxk::TileDims t = n->net.tile();
        if (nb < 1 || nb > n->net.max_batch()) return set_err(FX_INVALID_ARGUMENT, "fx_net_forward: batch out of range");
        if (!sigmoid && (channel < 0 || channel >= n->net.classes()))
            return set_err(FX_INVALID_ARGUMENT, "fx_net_forward: channel out of range");
        // The nb tiles are stacked along z: tile b is the volume's z-range [b tz, (b+1) tz).
        std::vector<fxk::TileOrigin> org(nb);
        for (int b = 0; b < nb; ++b) org[b] = {static_cast<int64_t>(b) * t.z, 0, 0};
        fxk::TileOrigin* d_org = nullptr;
        if (cudaMalloc(&d_org, sizeof(fxk::TileOrigin) * nb) != cudaSuccess)
            return set_err(FX_INTERNAL, "cudaMalloc failed");
        cudaMemcpyAsync(d_org, org.data(), sizeof(fxk::TileOrigin) * nb, cudaMemcpyHostToDevice, s);
        fxh::Status st = n->net.forward(dev_tiles, static_cast<int64_t>(nb) * t.z, t.y, t.x, d_org, nb, channel, sigmoid,
                                        nullptr, dev_prob, false, s);
        cudaError_t e = cudaStreamSynchronize(s);
        cudaFree(d_org);
        if (!st.ok()) return set_err(st);
        if (e != cudaSuccess) return set_err(fxh::cuda_status(e, "forward"));
        if ((st = n->net.take_device_status()).code) return set_err(st);
        return FX_OK;
    });
}

fx_status fx_predict_volume_dev(fx_net* n, const uint8_t* dev_vol, int64_t dz, int64_t dy, int64_t dx,
                                const fx_infer_opts* o, float* dev_prob, uint8_t* dev_u8, void* stream) {
    return guarded([&]() -> fx_status {
        if (!n || !dev_vol || !o || (!dev_prob && !dev_u8))
            return set_err(FX_INVALID_ARGUMENT, "fx_predict_volume_dev: null argument");
        if (dz < 1 || dy < 1 || dx < 1) return set_err(FX_INVALID_ARGUMENT, "fx_predict_volume_dev: empty volume");
        fxk::TileDims tl{};
        if (fx_status r = fxh::opts_tile(o, &tl)) return r;
        cudaSetDevice(n->net.device());
        const int64_t d[3] = {dz, dy, dx};
        int64_t co[3], ce[3];
        fxh::crop_box(o, d, co, ce);
        float* acc = dev_prob;
        if (!acc) {
            const size_t no = static_cast<size_t>(std::max<int64_t>(ce[0], 1)) * std::max<int64_t>(ce[1], 1) *
                              std::max<int64_t>(ce[2], 1);
            uint8_t* unused = nullptr;
            fxh::Status st = n->net.workspace(0, no * sizeof(float), 0, &unused, &acc, nullptr);
            if (!st.ok()) return set_err(st);
        }
        return fxh::predict_resident(n, dev_vol, dz, dy, dx, o, acc, dev_prob, dev_u8,
                                     static_cast<cudaStream_t>(stream), false);
    });
}

fx_status fx_predict_tiles_dev(fx_net* n, const uint8_t* dev_slab, int64_t slab_dz, int64_t dy, int64_t dx,
                               int64_t z_origin, int64_t full_dz, const fx_infer_opts* o, int64_t tile_begin,
                               int64_t tile_end, float* dev_acc, void* stream) {
    return guarded([&]() -> fx_status {
        if (!n || !dev_slab || !o || !dev_acc) return set_err(FX_INVALID_ARGUMENT, "fx_predict_tiles_dev: null argument");
        if (slab_dz < 1 || dy < 1 || dx < 1 || full_dz < slab_dz || z_origin < 0 || z_origin + slab_dz > full_dz)
            return set_err(FX_INVALID_ARGUMENT, "fx_predict_tiles_dev: bad slab geometry");
        fxk::TileDims tl{};
        if (fx_status r = fxh::opts_tile(o, &tl)) return r;
        cudaSetDevice(n->net.device());
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : n->net.stream();
        fxh::RunOpts ro = fxh::run_opts(o);
        if (ro.core_org[0] || ro.core_org[1] || ro.core_org[2] || ro.core_ext[0] > 0 || ro.core_ext[1] > 0 ||
            ro.core_ext[2] > 0)
            return set_err(FX_UNSUPPORTED, "fx_predict_tiles_dev: output crops are taken by fx_predict_volume only");
        fxh::Status st = n->net.predict_tiles(dev_slab, slab_dz, dy, dx, z_origin, full_dz, tl, o->overlap,
                                              o->channel, o->sigmoid, o->batch, tile_begin, tile_end, dev_acc, s, 0,
                                              -1, o->tta, ro);
        return st.ok() ? FX_OK : set_err(st);
    });
}

fx_status fx_net_device_status(fx_net* n) {
    return guarded([&]() -> fx_status {
        if (!n) return set_err(FX_INVALID_ARGUMENT, "fx_net_device_status: null net");
        fxh::Status st = n->net.take_device_status();
        return st.ok() ? FX_OK : set_err(st);
    });
}

fx_status fx_selftest_wait_timeout(int device, uint64_t wait_ns, uint32_t* status_out) {
    return guarded([&]() -> fx_status {
        if (!status_out || wait_ns == 0) return set_err(FX_INVALID_ARGUMENT, "fx_selftest_wait_timeout: bad argument");
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
            return set_err(FX_INVALID_ARGUMENT, "fx_selftest_wait_timeout: no such device");
        cudaSetDevice(device);
        if (!is_sm100()) return set_err(FX_UNSUPPORTED, "fx_selftest_wait_timeout: needs an sm_100 GPU");
        // one small stride-1 f16 conv (16 -> 128 channels over 8^3: the kernel's regular program)
        fxh::Layer L;
        L.name = "selftest";
        L.kind = fxh::Layer::kConv;
        L.Cin = 16;
        L.Cout = 128;
        L.stride = 1;
        L.w.assign(static_cast<size_t>(L.Cout) * L.Cin * 27, 0.f);
        const fxh::ActGeom g{8, 8, 8};
        std::vector<void*> allocs;
        struct Free {
            std::vector<void*>& a;
            ~Free() {
                for (void* p : a) cudaFree(p);
            }
        } fr{allocs};
        const int sms = sm_count_of_current();
        fxh::Status st = fxh::build_layer_program(L, fxk::kOpF16, g, g, 1, sms, allocs);
        if (!st.ok()) return set_err(st);
        Scratch sc;
        const int64_t igs = g.gs(), ibs = (L.Cin / 8) * igs, obs = (L.Cout / 8) * igs;
        const int64_t nrec = std::max<int64_t>((g.rows() + 125) / 126, sms) * fxk::kStatRecsPerUnit;
        auto* in = static_cast<uint8_t*>(sc.get(static_cast<size_t>(ibs)));
        auto* out = static_cast<uint8_t*>(sc.get(static_cast<size_t>(obs)));
        L.d_partials = static_cast<float*>(sc.get(sizeof(float) * nrec * L.Cout * 2));
        L.nrec_cap = nrec;
        auto* d_status = static_cast<uint32_t*>(sc.get(sizeof(uint32_t)));
        if (!in || !out || !L.d_partials || !d_status) return set_err(FX_INTERNAL, "cudaMalloc failed");
        cudaStream_t s = nullptr;
        cudaMemsetAsync(in, 0, static_cast<size_t>(ibs), s);
        cudaMemsetAsync(L.d_partials, 0, sizeof(float) * nrec * L.Cout * 2, s);
        cudaMemsetAsync(d_status, 0, sizeof(uint32_t), s);
        st = fxh::launch_layer(L, fxk::kOpF16, g, g, in, ibs, igs, out, obs, igs, 0, 1.f, nullptr, 1, sms, d_status, s,
                               true, wait_ns, 1);
        if (!st.ok()) return set_err(st);
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return set_err(fxh::cuda_status(e, "fx_selftest_wait_timeout"));
        uint32_t v = 0;
        if ((e = cudaMemcpy(&v, d_status, 4, cudaMemcpyDeviceToHost)) != cudaSuccess)
            return set_err(fxh::cuda_status(e, "fx_selftest_wait_timeout"));
        *status_out = v;
        return FX_OK;
    });
}

fx_status fx_accum_add(float* dev_dst, const float* dev_src, int64_t n, void* stream) {
    return guarded([&]() -> fx_status {
        if (!dev_dst || !dev_src || n < 0) return set_err(FX_INVALID_ARGUMENT, "fx_accum_add: bad argument");
        cudaError_t e = fxk::launch_accum_add(dev_dst, dev_src, n, static_cast<cudaStream_t>(stream));
        return e == cudaSuccess ? FX_OK : set_err(fxh::cuda_status(e, "fx_accum_add"));
    });
}

fx_status fx_predict_volume(fx_net* n, const uint8_t* host_vol, int64_t dz, int64_t dy, int64_t dx,
                            const fx_infer_opts* o, float* host_prob, uint8_t* host_u8) {
    return guarded([&]() -> fx_status {
        if (!n || !host_vol || !o) return set_err(FX_INVALID_ARGUMENT, "fx_predict_volume: null argument");
        if (dz < 1 || dy < 1 || dx < 1) return set_err(FX_INVALID_ARGUMENT, "fx_predict_volume: empty volume");
        fxk::TileDims tl{};  // the reference's patch % 64 check (src/ml/infer.hpp:459) for cubes
        if (fx_status r = fxh::opts_tile(o, &tl)) return r;
        cudaSetDevice(n->net.device());
        cudaStream_t s = n->net.stream();
        const size_t nv = static_cast<size_t>(dz) * dy * dx;
        const int64_t d[3] = {dz, dy, dx};
        int64_t co[3], ce[3];
        fxh::crop_box(o, d, co, ce);
        const size_t no = static_cast<size_t>(std::max<int64_t>(ce[0], 0)) * std::max<int64_t>(ce[1], 0) *
                          std::max<int64_t>(ce[2], 0);  // output voxels
        uint8_t *d_vol = nullptr, *d_u8 = nullptr;
        float* d_acc = nullptr;
        fxh::Status st = n->net.workspace(nv, std::max<size_t>(no, 1) * sizeof(float), host_u8 ? std::max<size_t>(no, 1) : 0,
                                          &d_vol, &d_acc, &d_u8);
        if (!st.ok()) return set_err(st);
        cudaMemcpyAsync(d_vol, host_vol, nv, cudaMemcpyHostToDevice, s);
        // the normalised probability overwrites the accumulator in place
        float* d_prob = host_prob ? d_acc : nullptr;
        if (fx_status r = fxh::predict_resident(n, d_vol, dz, dy, dx, o, d_acc, d_prob, host_u8 ? d_u8 : nullptr))
            return r;
        if (host_prob) cudaMemcpyAsync(host_prob, d_prob, no * sizeof(float), cudaMemcpyDeviceToHost, s);
        if (host_u8) cudaMemcpyAsync(host_u8, d_u8, no, cudaMemcpyDeviceToHost, s);
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return set_err(fxh::cuda_status(e, "predict_volume"));
        return FX_OK;
    });
}

fx_status fx_net_profile(fx_net* n, int enable) {
    if (!n) return set_err(FX_INVALID_ARGUMENT, "fx_net_profile: null net");
    n->net.profile(enable != 0);
    return FX_OK;
}

fx_status fx_net_profile_read(fx_net* n, double* conv_ms, double* conv_flops, double* fp8_flops,
                              int64_t* conv_launches, double* per_launch, int cap) {
    return guarded([&]() -> fx_status {
        if (!n) return set_err(FX_INVALID_ARGUMENT, "fx_net_profile_read: null net");
        fxh::Net::ProfileTotals t;
        fxh::Status st = n->net.profile_read(t, per_launch, cap);
        if (!st.ok()) return set_err(st);
        if (conv_ms) *conv_ms = t.conv_ms;
        if (conv_flops) *conv_flops = t.conv_flops;
        if (fp8_flops) *fp8_flops = t.fp8_flops;
        if (conv_launches) *conv_launches = t.conv_launches;
        return FX_OK;
    });
}

int fx_net_profile_read_layers(fx_net* n, double* layer_ms, int cap) {
    int out = -1;
    const fx_status r = guarded([&]() -> fx_status {
        if (!n) return set_err(FX_INVALID_ARGUMENT, "fx_net_profile_read_layers: null net");
        fxh::Net::ProfileTotals t;
        std::vector<double> per;
        fxh::Status st = n->net.profile_read(t, nullptr, 0, &per);
        if (!st.ok()) return set_err(st);
        for (int i = 0; layer_ms && i < cap && i < static_cast<int>(per.size()); ++i) layer_ms[i] = per[i];
        out = static_cast<int>(per.size());
        return FX_OK;
    });
    return r == FX_OK ? out : -1;
}

unsigned long long fx_kernel_launches(void) { return fxk::launch_count(); }

void fx_conv_trace_buffer(void* dev_counters) { fxh::g_conv_trace = static_cast<unsigned long long*>(dev_counters); }

int64_t fx_tile_starts(int64_t dim, int patch, double overlap, int64_t* out, int64_t cap) {
    const auto v = fenix::ml::tile_starts(dim, patch, overlap);
    for (int64_t i = 0; i < cap && i < static_cast<int64_t>(v.size()); ++i) out[i] = v[static_cast<size_t>(i)];
    return static_cast<int64_t>(v.size());
}

void fx_gaussian1d(int n, float* out) {
    const auto v = fenix::ml::gaussian1d(n);
    std::copy(v.begin(), v.end(), out);
}

void fx_weight_profile(const float* g, int patch, const int64_t* starts, int64_t nstarts, int64_t c0, int64_t cn,
                       int64_t dim, float* out) {
    std::vector<float> gv(g, g + patch);
    std::vector<int64_t> sv(starts, starts + nstarts);
    const auto w = fenix::ml::weight_profile(gv, sv, c0, cn, dim, patch);
    std::copy(w.begin(), w.end(), out);
}

fx_status fx_norm_tiles(const uint8_t* dev_vol, int64_t dz, int64_t dy, int64_t dx, const int64_t* host_origins,
                        int ntiles, int patch, float* dev_out, void* stream) {
    return guarded([&]() -> fx_status {
        if (!dev_vol || !host_origins || !dev_out || ntiles < 1 || patch < 1)
            return set_err(FX_INVALID_ARGUMENT, "fx_norm_tiles: bad argument");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Scratch sc;
        std::vector<fxk::TileOrigin> org(ntiles);
        for (int i = 0; i < ntiles; ++i) org[i] = {host_origins[3 * i], host_origins[3 * i + 1], host_origins[3 * i + 2]};
        auto* d_org = static_cast<fxk::TileOrigin*>(sc.get(sizeof(fxk::TileOrigin) * ntiles));
        auto* d_sums = static_cast<unsigned long long*>(sc.get(sizeof(unsigned long long) * 2 * ntiles));
        if (!d_org || !d_sums) return set_err(FX_INTERNAL, "cudaMalloc failed");
        cudaMemcpyAsync(d_org, org.data(), sizeof(fxk::TileOrigin) * ntiles, cudaMemcpyHostToDevice, s);
        cudaMemsetAsync(d_sums, 0, sizeof(unsigned long long) * 2 * ntiles, s);
        cudaError_t e = fxk::launch_tile_sums(dev_vol, dz, dy, dx, d_org, ntiles, fxk::TileDims{patch, patch, patch}, d_sums, s);
        if (e == cudaSuccess)
            e = fxk::launch_tile_norm(dev_vol, dz, dy, dx, d_org, ntiles, fxk::TileDims{patch, patch, patch}, d_sums, nullptr, 0, 0, fxk::kOpF16,
                                      dev_out, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        return e == cudaSuccess ? FX_OK : set_err(fxh::cuda_status(e, "fx_norm_tiles"));
    });
}

fx_status fx_norm_tiles_mode(const uint8_t* dev_vol, int64_t dz, int64_t dy, int64_t dx, const int64_t* host_origins,
                             int ntiles, int patch, int norm, float* dev_out, void* stream) {
    return guarded([&]() -> fx_status {
        if (!dev_vol || !host_origins || !dev_out || ntiles < 1 || ntiles > 65535 || patch < 1 || norm < 0 || norm > 2)
            return set_err(FX_INVALID_ARGUMENT, "fx_norm_tiles_mode: bad argument");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Scratch sc;
        std::vector<fxk::TileOrigin> org(ntiles);
        for (int i = 0; i < ntiles; ++i) org[i] = {host_origins[3 * i], host_origins[3 * i + 1], host_origins[3 * i + 2]};
        auto* d_org = static_cast<fxk::TileOrigin*>(sc.get(sizeof(fxk::TileOrigin) * ntiles));
        auto* d_sums = static_cast<unsigned long long*>(sc.get(sizeof(unsigned long long) * 2 * ntiles));
        auto* d_hist = static_cast<unsigned*>(sc.get(sizeof(unsigned) * 256 * ntiles));
        auto* d_lut = static_cast<float*>(sc.get(sizeof(float) * 256 * ntiles));
        if (!d_org || !d_sums || !d_hist || !d_lut) return set_err(FX_INTERNAL, "cudaMalloc failed");
        cudaMemcpyAsync(d_org, org.data(), sizeof(fxk::TileOrigin) * ntiles, cudaMemcpyHostToDevice, s);
        cudaMemsetAsync(d_sums, 0, sizeof(unsigned long long) * 2 * ntiles, s);
        cudaMemsetAsync(d_hist, 0, sizeof(unsigned) * 256 * ntiles, s);
        cudaError_t e = fxk::launch_tile_sums(dev_vol, dz, dy, dx, d_org, ntiles, fxk::TileDims{patch, patch, patch}, d_sums, s, d_hist);
        const int64_t n = static_cast<int64_t>(patch) * patch * patch;
        if (e == cudaSuccess) e = fxk::launch_tile_lut(d_sums, d_hist, ntiles, n, norm, d_lut, nullptr, s);
        if (e == cudaSuccess)
            e = fxk::launch_tile_norm(dev_vol, dz, dy, dx, d_org, ntiles, fxk::TileDims{patch, patch, patch}, d_sums, nullptr, 0, 0, fxk::kOpF16,
                                      dev_out, s, nullptr, d_lut);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        return e == cudaSuccess ? FX_OK : set_err(fxh::cuda_status(e, "fx_norm_tiles_mode"));
    });
}

fx_status fx_conv3d(const float* dev_x, int B, int Cin, int D, int H, int W, const float* dev_w, int Cout, int stride,
                    fx_precision precision, float* dev_y, float* dev_stats, void* stream) {
    return guarded([&]() -> fx_status {
        if (!dev_x || !dev_w || !dev_y || B < 1 || Cin < 1 || Cout < 1 || D < 1 || H < 1 || W < 1)
            return set_err(FX_INVALID_ARGUMENT, "fx_conv3d: bad argument");
        if (stride != 1 && stride != 2) return set_err(FX_INVALID_ARGUMENT, "fx_conv3d: stride must be 1 or 2");
        if (stride == 2 && (D % 2 || H % 2 || W % 2)) return set_err(FX_INVALID_ARGUMENT, "fx_conv3d: stride 2 needs even extents");
        if (precision < FX_PREC_BF16 || precision > FX_PREC_F16) return set_err(FX_INVALID_ARGUMENT, "fx_conv3d: bad precision");
        const int q = static_cast<int>(precision);  // fx_precision values are the kernel's operand types
        const bool fp8 = q == fxk::kOpE4M3;
        if (Cin == 1 && (stride != 1 || fp8)) return set_err(FX_UNSUPPORTED, "fx_conv3d: 1-channel input is 16-bit stride 1");
        if (Cout % 16) return set_err(FX_UNSUPPORTED, "fx_conv3d: Cout must be a multiple of 16");
        if (!is_sm100()) return set_err(FX_UNSUPPORTED, "fx_conv3d: needs an sm_100 GPU");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Scratch sc;
        fxh::Layer L;
        L.name = "fx_conv3d";
        L.kind = Cin == 1 ? fxh::Layer::kFirst : fxh::Layer::kConv;
        L.Cin = Cin;
        L.Cout = Cout;
        L.stride = stride;
        L.smask = stride == 2 ? 7 : 0;
        L.w.resize(static_cast<size_t>(Cout) * Cin * 27);
        cudaMemcpyAsync(L.w.data(), dev_w, L.w.size() * sizeof(float), cudaMemcpyDeviceToHost, s);
        cudaStreamSynchronize(s);
        const int cg = fp8 ? 16 : 8;
        if (Cin > 1 && Cin % (2 * cg)) return set_err(FX_UNSUPPORTED, "fx_conv3d: Cin must be a multiple of 16 (bf16) / 32 (fp8)");
        const fxh::ActGeom gin{D, H, W};
        const fxh::ActGeom gout{D / stride, H / stride, W / stride};
        const int64_t vin = static_cast<int64_t>(D) * H * W;
        if (fp8) L.in_scale = std::max(device_absmax(dev_x, vin * B * Cin, s, sc), 1e-8f) / 448.f;
        std::vector<void*> allocs;
        struct Free {
            std::vector<void*>& a;
            ~Free() {
                for (void* p : a) cudaFree(p);
            }
        } fr{allocs};
        fxh::Status st = fxh::build_layer_program(L, q, gin, gout, B, sm_count_of_current(), allocs);
        if (!st.ok()) return set_err(st);
        // input in the kernel's layout
        uint8_t* in;
        int64_t ibs, igs;
        if (L.kind == fxh::Layer::kFirst) {
            igs = gin.gs();
            ibs = 2 * igs;
            in = static_cast<uint8_t*>(sc.get(static_cast<size_t>(B) * ibs));
            if (!in) return set_err(FX_INTERNAL, "cudaMalloc failed");
            cudaMemsetAsync(in, 0, static_cast<size_t>(B) * ibs, s);
            fxk::launch_pack_first(dev_x, B, D, H, W, in, ibs, igs, q, s);
        } else if (stride == 1) {
            igs = gin.gs();
            ibs = (Cin / cg) * igs;
            in = static_cast<uint8_t*>(sc.get(static_cast<size_t>(B) * ibs));
            if (!in) return set_err(FX_INTERNAL, "cudaMalloc failed");
            cudaMemsetAsync(in, 0, static_cast<size_t>(B) * ibs, s);
            fxk::launch_pack(dev_x, B, Cin, D, H, W, in, ibs, igs, q, fp8 ? 1.f / L.in_scale : 1.f, 0, 0, 0, 0, s);
        } else {
            const int64_t ps = gout.gs();
            igs = 8 * ps;
            ibs = (Cin / cg) * igs;
            in = static_cast<uint8_t*>(sc.get(static_cast<size_t>(B) * ibs));
            if (!in) return set_err(FX_INTERNAL, "cudaMalloc failed");
            cudaMemsetAsync(in, 0, static_cast<size_t>(B) * ibs, s);
            fxk::launch_pack(dev_x, B, Cin, D, H, W, in, ibs, igs, q, fp8 ? 1.f / L.in_scale : 1.f, 7, gout.H + 2,
                             gout.W + 2, ps, s);
        }
        const int64_t ogs = gout.gs(), obs = (Cout / 8) * ogs;
        auto* out = static_cast<uint8_t*>(sc.get(static_cast<size_t>(B) * obs));
        const int64_t rows = static_cast<int64_t>(gout.D) * (gout.H + 2) * (gout.W + 2);
        const int64_t nrec = std::max<int64_t>((rows + 125) / 126, sm_count_of_current()) * fxk::kStatRecsPerUnit;
        L.d_partials = static_cast<float*>(sc.get(sizeof(float) * B * nrec * Cout * 2));
        L.nrec_cap = nrec;
        auto* d_status = static_cast<uint32_t*>(sc.get(sizeof(uint32_t)));
        if (!out || !L.d_partials || !d_status) return set_err(FX_INTERNAL, "cudaMalloc failed");
        cudaMemsetAsync(L.d_partials, 0, sizeof(float) * B * nrec * Cout * 2, s);  // the epilogue adds into it
        cudaMemsetAsync(out, 0, static_cast<size_t>(B) * obs, s);
        cudaMemsetAsync(d_status, 0, sizeof(uint32_t), s);
        st = fxh::launch_layer(L, q, gin, gout, in, ibs, igs, out, obs, ogs, 0, 1.f, nullptr, B, sm_count_of_current(),
                               d_status, s, /*per_column=*/true);
        if (!st.ok()) return set_err(st);
        fxk::launch_unpack(out, obs, ogs, fxk::kOpF16, 1.f, B, Cout, gout.D, gout.H, gout.W, dev_y, s);
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return set_err(fxh::cuda_status(e, "fx_conv3d"));
        uint32_t status = 0;
        cudaMemcpy(&status, d_status, 4, cudaMemcpyDeviceToHost);
        if (status) return set_err(FX_INTERNAL, "fx_conv3d: device status " + std::to_string(status));
        if (dev_stats) {
            std::vector<float> part(static_cast<size_t>(B) * L.nrec * Cout * 2);
            cudaMemcpy(part.data(), L.d_partials, part.size() * sizeof(float), cudaMemcpyDeviceToHost);
            std::vector<float> res(static_cast<size_t>(B) * Cout * 2);
            const double cnt = static_cast<double>(gout.D) * gout.H * gout.W;
            for (int b = 0; b < B; ++b)
                for (int c = 0; c < Cout; ++c) {
                    double a1 = 0, a2 = 0;
                    for (int r = 0; r < L.nrec; ++r) {
                        a1 += part[((static_cast<size_t>(b) * L.nrec + r) * Cout + c) * 2];
                        a2 += part[((static_cast<size_t>(b) * L.nrec + r) * Cout + c) * 2 + 1];
                    }
                    const double m = a1 / cnt;
                    res[(static_cast<size_t>(b) * Cout + c) * 2] = static_cast<float>(m);
                    res[(static_cast<size_t>(b) * Cout + c) * 2 + 1] = static_cast<float>(a2 / cnt - m * m);
                }
            cudaMemcpy(dev_stats, res.data(), res.size() * sizeof(float), cudaMemcpyHostToDevice);
        }
        return FX_OK;
    });
}

fx_status fx_conv_transpose2(const float* dev_x, int B, int Cin, int D, int H, int W, const float* dev_w,
                             const float* dev_bias, int Cout, fx_precision precision, float* dev_y, void* stream) {
    return guarded([&]() -> fx_status {
        if (!dev_x || !dev_w || !dev_bias || !dev_y || B < 1 || Cin < 1 || Cout < 1 || D < 1 || H < 1 || W < 1)
            return set_err(FX_INVALID_ARGUMENT, "fx_conv_transpose2: bad argument");
        if (!is_sm100()) return set_err(FX_UNSUPPORTED, "fx_conv_transpose2: needs an sm_100 GPU");
        if (precision < FX_PREC_BF16 || precision > FX_PREC_F16)
            return set_err(FX_INVALID_ARGUMENT, "fx_conv_transpose2: bad precision");
        const int q = static_cast<int>(precision);
        const bool fp8 = q == fxk::kOpE4M3;
        const int cg = fp8 ? 16 : 8;
        if (Cin % (2 * cg) || Cout % 16)
            return set_err(FX_UNSUPPORTED, "fx_conv_transpose2: channel counts not supported");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Scratch sc;
        fxh::Layer L;
        L.name = "fx_conv_transpose2";
        L.kind = fxh::Layer::kUp;
        L.Cin = Cin;
        L.Cout = Cout;
        L.stride = 2;
        L.smask = 7;
        L.w.resize(static_cast<size_t>(Cin) * Cout * 8);
        L.b.resize(Cout);
        cudaMemcpyAsync(L.w.data(), dev_w, L.w.size() * sizeof(float), cudaMemcpyDeviceToHost, s);
        cudaMemcpyAsync(L.b.data(), dev_bias, L.b.size() * sizeof(float), cudaMemcpyDeviceToHost, s);
        cudaStreamSynchronize(s);
        const fxh::ActGeom gin{D, H, W}, gout{2 * D, 2 * H, 2 * W};
        const int64_t vin = static_cast<int64_t>(D) * H * W;
        if (fp8) L.in_scale = std::max(device_absmax(dev_x, vin * B * Cin, s, sc), 1e-8f) / 448.f;
        std::vector<void*> allocs;
        struct Free {
            std::vector<void*>& a;
            ~Free() {
                for (void* p : a) cudaFree(p);
            }
        } fr{allocs};
        fxh::Status st = fxh::build_layer_program(L, q, gin, gout, B, sm_count_of_current(), allocs);
        if (!st.ok()) return set_err(st);
        const int64_t igs = gin.gs(), ibs = (Cin / cg) * igs;
        const int64_t ogs = gout.gs(), obs = (Cout / 8) * ogs;  // output cells are bf16 here
        auto* in = static_cast<uint8_t*>(sc.get(static_cast<size_t>(B) * ibs));
        auto* out = static_cast<uint8_t*>(sc.get(static_cast<size_t>(B) * obs));
        auto* d_status = static_cast<uint32_t*>(sc.get(sizeof(uint32_t)));
        auto* d_amax = static_cast<unsigned*>(sc.get(sizeof(unsigned)));
        if (!in || !out || !d_status || !d_amax) return set_err(FX_INTERNAL, "cudaMalloc failed");
        cudaMemsetAsync(in, 0, static_cast<size_t>(B) * ibs, s);
        cudaMemsetAsync(out, 0, static_cast<size_t>(B) * obs, s);
        cudaMemsetAsync(d_status, 0, sizeof(uint32_t), s);
        fxk::launch_pack(dev_x, B, Cin, D, H, W, in, ibs, igs, q, fp8 ? 1.f / L.in_scale : 1.f, 0, 0, 0, 0, s);
        // This entry point writes f16 output cells whatever the operand type (an e4m3 output
        // would need its scale before the run).
        st = fxh::launch_layer(L, q, gin, gout, in, ibs, igs, out, obs, ogs, fxk::kOpF16, 1.f, d_amax, B,
                               sm_count_of_current(), d_status, s);
        if (!st.ok()) return set_err(st);
        fxk::launch_unpack(out, obs, ogs, fxk::kOpF16, 1.f, B, Cout, gout.D, gout.H, gout.W, dev_y, s);
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return set_err(fxh::cuda_status(e, "fx_conv_transpose2"));
        uint32_t status = 0;
        cudaMemcpy(&status, d_status, 4, cudaMemcpyDeviceToHost);
        if (status) return set_err(FX_INTERNAL, "fx_conv_transpose2: device status " + std::to_string(status));
        return FX_OK;
    });
}

fx_status fx_accum_finalize(const float* dev_acc, int64_t dz, int64_t dy, int64_t dx, int64_t z_begin, int64_t z_end,
                            const float* dev_wz, const float* dev_wy, const float* dev_wx, float* dev_prob,
                            uint8_t* dev_u8, void* stream) {
    return guarded([&]() -> fx_status {
        if (!dev_acc || !dev_wz || !dev_wy || !dev_wx || z_begin < 0 || z_end > dz || z_begin > z_end)
            return set_err(FX_INVALID_ARGUMENT, "fx_accum_finalize: bad argument");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cudaError_t e =
            fxk::launch_accum_finalize(dev_acc, dz, dy, dx, z_begin, z_end, dev_wz, dev_wy, dev_wx, dev_prob, dev_u8, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        return e == cudaSuccess ? FX_OK : set_err(fxh::cuda_status(e, "fx_accum_finalize"));
    });
}


fx_status fx_norm_tiles_noalloc(const uint8_t* dev_vol, int64_t dz, int64_t dy, int64_t dx,
                                const int64_t* host_origins, int ntiles, int patch, float* dev_out, void* stream) {
    return guarded([&]() -> fx_status {
        if (!dev_vol || !host_origins || !dev_out || ntiles < 1 || patch < 1 || dz < 1 || dy < 1 || dx < 1)
            return set_err(FX_INVALID_ARGUMENT, "fx_norm_tiles_noalloc: bad argument");
        if (ntiles > kNoAllocMaxTiles)
            return set_err(FX_INVALID_ARGUMENT, "fx_norm_tiles_noalloc: " + std::to_string(ntiles) +
                                                    " tiles exceed the static scratch limit of " +
                                                    std::to_string(kNoAllocMaxTiles) + " tiles per call");
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return set_err(fxh::cuda_status(e, "fx_norm_tiles_noalloc: cudaGetDevice"));
        if (dev < 0 || dev >= kNoAllocMaxDevices)
            return set_err(FX_UNSUPPORTED, "fx_norm_tiles_noalloc: device index beyond 63");
        // Set-up, once per device with that device current: the first call on a device resolves
        // the scratch's address there.
        static std::mutex mu;
        static unsigned char* base_of[kNoAllocMaxDevices] = {};
        unsigned char* base;
        {
            std::lock_guard<std::mutex> lock(mu);
            if (!base_of[dev]) {
                void* p = nullptr;
                e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
                if (e != cudaSuccess || !p)
                    return set_err(fxh::cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                                                    "fx_norm_tiles_noalloc: cudaGetSymbolAddress"));
                base_of[dev] = static_cast<unsigned char*>(p);
            }
            base = base_of[dev];
        }
        auto* org = reinterpret_cast<fxk::TileOrigin*>(base);
        auto* sums = reinterpret_cast<unsigned long long*>(base + kNoAllocOrgBytes);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        e = cudaMemcpyAsync(org, host_origins, sizeof(fxk::TileOrigin) * ntiles, cudaMemcpyHostToDevice, s);
        // the sums are accumulated with atomics: they start at zero on every call
        if (e == cudaSuccess) e = cudaMemsetAsync(sums, 0, 2 * sizeof(unsigned long long) * ntiles, s);
        if (e == cudaSuccess) e = fxk::launch_tile_sums(dev_vol, dz, dy, dx, org, ntiles, fxk::TileDims{patch, patch, patch}, sums, s);
        if (e == cudaSuccess)
            e = fxk::launch_tile_norm(dev_vol, dz, dy, dx, org, ntiles, fxk::TileDims{patch, patch, patch}, sums, nullptr, 0, 0, fxk::kOpF16, dev_out,
                                      s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        return e == cudaSuccess ? FX_OK : set_err(fxh::cuda_status(e, "fx_norm_tiles_noalloc"));
    });
}

}  // extern "C"
