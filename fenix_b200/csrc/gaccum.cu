// gaccum.cu — the global-grid accumulator of predict-scroll (GlobalAccum,
// src/ml/global_accum.hpp:37-198) on the device, with its z-sweep finalize and resume floor.
//
// The reference keeps a sparse map of 64^3 f32 blocks in host memory. Here the accumulator is a
// dense window of f32 planes in HBM that slides down the bbox: it always starts at the finalize
// floor (a multiple of 64 planes), tiles scatter into it with atomics, and finalizing chunk rows
// below a limit normalises them by the factorised profile (Wz.Wy.Wx), encodes u8, copies them to
// the host and moves the window down (the planes still live are copied to the second window
// buffer). A volume larger than HBM streams through: input planes per tile row, u8 per chunk row.
#include "fenix_b200.h"
#include "eltwise.cuh"
#include "fenix_b200/ml/tiling.hpp"
#include "net.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <memory>
#include <new>
#include <string>
#include <vector>

namespace fxh {
fx_status abi_error(int code, const std::string& msg);  // capi.cu: sets the thread's last error
fx_status abi_exception();                              // capi.cu: status + message of a caught exception
}
// No exception crosses the C ABI.
#define FX_ABI_TRY try {
#define FX_ABI_CATCH \
    }                \
    catch (...) {    \
        return fxh::abi_exception(); \
    }

struct fx_gaccum {
    static constexpr int64_t T = 64;  // chunk edge (GlobalAccum::T)
    int dev = 0;
    int64_t org[3] = {0, 0, 0}, ext[3] = {0, 0, 0};
    int P = 0;
    double overlap = 0.5;
    std::vector<int64_t> zs, ys, xs;
    float* d_g = nullptr;
    float* d_W[3] = {nullptr, nullptr, nullptr};
    float* win[2] = {nullptr, nullptr};
    int cur = 0;
    int64_t win_planes = 0;
    int64_t wz0 = 0;  // bbox-local plane of window plane 0 (= floor_row * T)
    int64_t floor_row = 0, ncz = 0;
    uint8_t* d_u8 = nullptr;
    uint8_t* d_slab = nullptr;
    float* d_prob = nullptr;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;

    ~fx_gaccum() {
        cudaSetDevice(dev);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : allocs) cudaFree(p);
        if (stream) cudaStreamDestroy(stream);
    }
    void* alloc(size_t bytes) {
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
        allocs.push_back(p);
        return p;
    }
    int64_t plane() const { return ext[1] * ext[2]; }
};

namespace {

using fxh::abi_error;

fx_status cuda_err(cudaError_t e, const char* what) {
    return abi_error(FX_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
}

// Move the window so that it starts at plane new_wz0 (>= wz0): live planes go to the other
// buffer, the rest of it is zeroed.
cudaError_t slide(fx_gaccum* a, int64_t new_wz0) {
    const int64_t shift = new_wz0 - a->wz0;
    if (shift <= 0) return cudaSuccess;
    const int64_t keep = std::max<int64_t>(0, a->win_planes - shift);
    const size_t pb = sizeof(float) * static_cast<size_t>(a->plane());
    float* src = a->win[a->cur];
    float* dst = a->win[a->cur ^ 1];
    cudaError_t e = cudaSuccess;
    if (keep > 0) e = cudaMemcpyAsync(dst, src + shift * a->plane(), keep * pb, cudaMemcpyDeviceToDevice, a->stream);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(dst + keep * a->plane(), 0, static_cast<size_t>(a->win_planes - keep) * pb, a->stream);
    a->cur ^= 1;
    a->wz0 = new_wz0;
    return e;
}

}  // namespace

extern "C" {

fx_status fx_gaccum_create(const int64_t* org, const int64_t* ext, int patch, double overlap, int64_t window_planes,
                           int device, fx_gaccum** out) {
    FX_ABI_TRY
    if (!org || !ext || !out || patch < 1 || !(overlap >= 0.0 && overlap < 1.0) || window_planes < 0)
        return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_create: bad argument");
    *out = nullptr;
    for (int i = 0; i < 3; ++i) {
        if (ext[i] < 1 || org[i] < 0) return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_create: bad bbox");
        if (org[i] % fx_gaccum::T)
            return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_create: bbox origin must be 64-aligned");
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n)
        return abi_error(FX_UNSUPPORTED, "fx_gaccum_create: no such CUDA device");
    cudaSetDevice(device);
    std::unique_ptr<fx_gaccum> a(new (std::nothrow) fx_gaccum);
    if (!a) return abi_error(FX_INTERNAL, "out of host memory");
    a->dev = device;
    for (int i = 0; i < 3; ++i) {
        a->org[i] = org[i];
        a->ext[i] = ext[i];
    }
    a->P = patch;
    a->overlap = overlap;
    a->zs = fenix::ml::tile_starts(ext[0], patch, overlap);
    a->ys = fenix::ml::tile_starts(ext[1], patch, overlap);
    a->xs = fenix::ml::tile_starts(ext[2], patch, overlap);
    a->ncz = (ext[0] + fx_gaccum::T - 1) / fx_gaccum::T;
    const std::vector<float> g = fenix::ml::gaussian1d(patch);
    const std::vector<int64_t>* st[3] = {&a->zs, &a->ys, &a->xs};
    int64_t wp = window_planes ? window_planes : patch + fx_gaccum::T;
    wp = (wp + fx_gaccum::T - 1) / fx_gaccum::T * fx_gaccum::T;
    a->win_planes = std::min<int64_t>(wp, a->ncz * fx_gaccum::T);
    cudaError_t e = cudaStreamCreateWithFlags(&a->stream, cudaStreamNonBlocking);
    a->d_g = static_cast<float*>(a->alloc(sizeof(float) * patch));
    for (int i = 0; i < 3; ++i) a->d_W[i] = static_cast<float*>(a->alloc(sizeof(float) * ext[i]));
    const size_t wbytes = sizeof(float) * static_cast<size_t>(a->win_planes) * a->plane();
    a->win[0] = static_cast<float*>(a->alloc(wbytes));
    a->win[1] = static_cast<float*>(a->alloc(wbytes));
    a->d_u8 = static_cast<uint8_t*>(a->alloc(static_cast<size_t>(a->win_planes) * a->plane()));
    a->d_prob = static_cast<float*>(a->alloc(sizeof(float) * static_cast<size_t>(patch) * patch * patch));
    bool ok = e == cudaSuccess && a->d_g && a->d_W[0] && a->d_W[1] && a->d_W[2] && a->win[0] && a->win[1] && a->d_u8 &&
              a->d_prob;
    if (ok) {
        e = cudaMemcpy(a->d_g, g.data(), sizeof(float) * patch, cudaMemcpyHostToDevice);
        for (int i = 0; i < 3 && e == cudaSuccess; ++i) {
            const std::vector<float> w = fenix::ml::weight_profile(g, *st[i], 0, ext[i], ext[i], patch);
            e = cudaMemcpy(a->d_W[i], w.data(), sizeof(float) * w.size(), cudaMemcpyHostToDevice);
        }
        if (e == cudaSuccess) e = cudaMemset(a->win[0], 0, wbytes);
        ok = e == cudaSuccess;
    }
    if (!ok) {
        return e != cudaSuccess ? cuda_err(e, "fx_gaccum_create") : abi_error(FX_INTERNAL, "fx_gaccum_create: cudaMalloc failed");
    }
    *out = a.release();
    return FX_OK;
    FX_ABI_CATCH
}

void fx_gaccum_destroy(fx_gaccum* a) { delete a; }

int64_t fx_gaccum_chunk_rows(const fx_gaccum* a) { return a ? a->ncz : 0; }
int64_t fx_gaccum_floor_row(const fx_gaccum* a) { return a ? a->floor_row : 0; }
int64_t fx_gaccum_window_planes(const fx_gaccum* a) { return a ? a->win_planes : 0; }
int64_t fx_gaccum_tile_rows(const fx_gaccum* a) { return a ? static_cast<int64_t>(a->zs.size()) : 0; }
int64_t fx_gaccum_row_start(const fx_gaccum* a, int64_t zi) {
    return (a && zi >= 0 && zi < static_cast<int64_t>(a->zs.size())) ? a->zs[static_cast<size_t>(zi)] : -1;
}

fx_status fx_gaccum_set_floor_row(fx_gaccum* a, int64_t floor_row) {
    FX_ABI_TRY
    if (!a) return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_set_floor_row: null accumulator");
    cudaSetDevice(a->dev);
    a->floor_row = std::clamp<int64_t>(floor_row, 0, a->ncz);
    // a fresh window at the new floor: nothing below it is accumulated any more
    a->wz0 = a->floor_row * fx_gaccum::T;
    const size_t wbytes = sizeof(float) * static_cast<size_t>(a->win_planes) * a->plane();
    cudaError_t e = cudaMemsetAsync(a->win[a->cur], 0, wbytes, a->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(a->stream);
    return e == cudaSuccess ? FX_OK : cuda_err(e, "fx_gaccum_set_floor_row");
    FX_ABI_CATCH
}

fx_status fx_gaccum_scatter(fx_gaccum* a, int64_t z0, int64_t y0, int64_t x0, const float* host_prob) {
    FX_ABI_TRY
    if (!a || !host_prob) return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_scatter: bad argument");
    cudaSetDevice(a->dev);
    const int64_t lz0 = z0 - a->org[0], ly0 = y0 - a->org[1], lx0 = x0 - a->org[2];
    const int64_t zhi = std::min<int64_t>(lz0 + a->P, a->ext[0]);
    if (zhi > a->wz0 + a->win_planes)
        return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_scatter: tile reaches beyond the accumulator window; "
                                              "finalize the rows below it first");
    const size_t n = static_cast<size_t>(a->P) * a->P * a->P;
    cudaError_t e = cudaMemcpyAsync(a->d_prob, host_prob, sizeof(float) * n, cudaMemcpyHostToDevice, a->stream);
    if (e == cudaSuccess)
        e = fxk::launch_scatter_tile(a->d_prob, a->P, lz0, ly0, lx0, a->ext[0], a->ext[1], a->ext[2],
                                     a->floor_row * fx_gaccum::T, a->d_g, a->win[a->cur], -a->wz0, a->win_planes,
                                     a->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(a->stream);  // host_prob may be reused on return
    return e == cudaSuccess ? FX_OK : cuda_err(e, "fx_gaccum_scatter");
    FX_ABI_CATCH
}

fx_status fx_gaccum_predict_row(fx_gaccum* a, fx_net* net, int64_t zi, const uint8_t* host_planes,
                                const fx_infer_opts* opts) {
    FX_ABI_TRY
    if (!a || !net || !host_planes || !opts || zi < 0 || zi >= static_cast<int64_t>(a->zs.size()))
        return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_predict_row: bad argument");
    if (opts->tile[0] || opts->tile[1] || opts->tile[2])
        return abi_error(FX_UNSUPPORTED, "fx_gaccum_predict_row: cubic tiles only (opts.tile must be 0)");
    if (opts->patch != a->P || opts->overlap != a->overlap)
        return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_predict_row: patch / overlap differ from the accumulator's");
    cudaSetDevice(a->dev);
    const int64_t z_lo = a->zs[static_cast<size_t>(zi)], z_hi = std::min<int64_t>(z_lo + a->P, a->ext[0]);
    if (z_hi > a->wz0 + a->win_planes)
        return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_predict_row: tile row reaches beyond the accumulator "
                                              "window; finalize the rows below it first");
    const size_t slab = static_cast<size_t>(z_hi - z_lo) * a->plane();
    if (!a->d_slab) {
        a->d_slab = static_cast<uint8_t*>(a->alloc(static_cast<size_t>(a->P) * a->plane()));
        if (!a->d_slab) return abi_error(FX_INTERNAL, "fx_gaccum_predict_row: cudaMalloc failed");
    }
    cudaError_t e = cudaMemcpyAsync(a->d_slab, host_planes, slab, cudaMemcpyHostToDevice, a->stream);
    if (e != cudaSuccess) return cuda_err(e, "fx_gaccum_predict_row: H2D");
    const int64_t per_row = static_cast<int64_t>(a->ys.size()) * static_cast<int64_t>(a->xs.size());
    fxh::Status st = net->net.predict_tiles(a->d_slab, z_hi - z_lo, a->ext[1], a->ext[2], z_lo, a->ext[0],
                                            fxk::TileDims{a->P, a->P, a->P}, opts->overlap, opts->channel, opts->sigmoid, opts->batch, zi * per_row,
                                            (zi + 1) * per_row, a->win[a->cur], a->stream, a->wz0, a->win_planes,
                                            opts->tta, fxh::run_opts(opts));
    if (!st.ok()) return abi_error(st.code, st.msg);
    e = cudaStreamSynchronize(a->stream);
    return e == cudaSuccess ? FX_OK : cuda_err(e, "fx_gaccum_predict_row");
    FX_ABI_CATCH
}

fx_status fx_gaccum_finalize_below(fx_gaccum* a, int64_t row_lim, uint8_t* host_u8, int64_t cap_bytes,
                                   int64_t* planes_out) {
    FX_ABI_TRY
    if (!a || !planes_out) return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_finalize_below: bad argument");
    cudaSetDevice(a->dev);
    *planes_out = 0;
    row_lim = std::min(row_lim, a->ncz);
    if (row_lim <= a->floor_row) return FX_OK;
    const int64_t z_begin = a->floor_row * fx_gaccum::T;
    const int64_t z_end = std::min(row_lim * fx_gaccum::T, a->ext[0]);
    const int64_t n = z_end - z_begin;
    if (n > a->win_planes) return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_finalize_below: more rows than the window holds");
    if (!host_u8 || cap_bytes < n * a->plane())
        return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_finalize_below: output buffer too small");
    cudaError_t e = fxk::launch_accum_finalize(a->win[a->cur], a->win_planes, a->ext[1], a->ext[2], 0, n,
                                               a->d_W[0] + a->wz0, a->d_W[1], a->d_W[2], nullptr, a->d_u8, a->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(host_u8, a->d_u8, static_cast<size_t>(n) * a->plane(), cudaMemcpyDeviceToHost, a->stream);
    if (e == cudaSuccess) e = slide(a, row_lim * fx_gaccum::T);
    if (e == cudaSuccess) e = cudaStreamSynchronize(a->stream);
    if (e != cudaSuccess) return cuda_err(e, "fx_gaccum_finalize_below");
    a->floor_row = row_lim;
    *planes_out = n;
    return FX_OK;
    FX_ABI_CATCH
}

// ---- composing accumulators of several GPUs (disjoint tile-row ranges, one accumulator each) ----

fx_status fx_gaccum_export_planes(fx_gaccum* a, int64_t z0, int64_t n, float* dev_dst) {
    FX_ABI_TRY
    if (!a || !dev_dst || n < 0) return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_export_planes: bad argument");
    if (z0 < a->wz0 || z0 + n > a->wz0 + a->win_planes)
        return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_export_planes: planes outside the accumulator window");
    cudaSetDevice(a->dev);
    const size_t pb = sizeof(float) * static_cast<size_t>(a->plane());
    cudaError_t e = cudaMemcpyAsync(dev_dst, a->win[a->cur] + (z0 - a->wz0) * a->plane(), static_cast<size_t>(n) * pb,
                                    cudaMemcpyDeviceToDevice, a->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(a->stream);
    return e == cudaSuccess ? FX_OK : cuda_err(e, "fx_gaccum_export_planes");
    FX_ABI_CATCH
}

fx_status fx_gaccum_add_planes(fx_gaccum* a, int64_t z0, int64_t n, const float* dev_src) {
    FX_ABI_TRY
    if (!a || !dev_src || n < 0) return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_add_planes: bad argument");
    if (z0 < a->wz0 || z0 + n > a->wz0 + a->win_planes)
        return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_add_planes: planes outside the accumulator window");
    cudaSetDevice(a->dev);
    cudaError_t e = fxk::launch_accum_add(a->win[a->cur] + (z0 - a->wz0) * a->plane(), dev_src, n * a->plane(), a->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(a->stream);
    return e == cudaSuccess ? FX_OK : cuda_err(e, "fx_gaccum_add_planes");
    FX_ABI_CATCH
}

fx_status fx_gaccum_discard_below(fx_gaccum* a, int64_t row_lim) {
    FX_ABI_TRY
    if (!a) return abi_error(FX_INVALID_ARGUMENT, "fx_gaccum_discard_below: null accumulator");
    cudaSetDevice(a->dev);
    row_lim = std::min(row_lim, a->ncz);
    if (row_lim <= a->floor_row) return FX_OK;
    cudaError_t e = slide(a, row_lim * fx_gaccum::T);
    if (e == cudaSuccess) e = cudaStreamSynchronize(a->stream);
    if (e != cudaSuccess) return cuda_err(e, "fx_gaccum_discard_below");
    a->floor_row = row_lim;
    return FX_OK;
    FX_ABI_CATCH
}

}  // extern "C"
