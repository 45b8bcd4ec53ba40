// multi.cu — one volume over several GPUs without a collective: z-slab sharding of the global tile
// grid, one host thread per GPU, tile-overlap bands folded into their owner over NVLink by a kernel
// that reads the neighbour's accumulator through peer memory, each GPU finalising the planes it owns.
//
// The reference runs one net replica per GPU on worker threads that claim tiles of one global grid
// and blend into a shared host accumulator (src/ml/inference.cpp:1129-1188 replicas, 1402-1586
// global mode). Here every GPU keeps its own accumulator window in HBM: tiles are independent
// forwards and the blend is a linear sum, so the only coupling is the sum over the planes where two
// GPUs' tiles overlap, at most one tile deep.
#include "fenix_b200.h"
#include "fenix_b200/ml/tiling.hpp"
#include "eltwise.cuh"
#include "net.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstring>
#include <exception>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace fxh {
fx_status abi_error(int code, const std::string& msg);
fx_status abi_exception();

// Contiguous near-equal ranges of the z-major tile list, one per shard; the input / accumulator slab
// of a shard holds every plane its tiles touch; the owned planes partition [0, dz).
std::vector<fx_shard> shard_plan(int64_t dz, int64_t dy, int64_t dx, int patch, double overlap, int n) {
    const auto zs = fenix::ml::tile_starts(dz, patch, overlap), ys = fenix::ml::tile_starts(dy, patch, overlap),
               xs = fenix::ml::tile_starts(dx, patch, overlap);
    const int64_t per_row = static_cast<int64_t>(ys.size()) * xs.size();
    const int64_t T = static_cast<int64_t>(zs.size()) * per_row;
    std::vector<fx_shard> out(static_cast<size_t>(n));
    int prev_live = -1;
    for (int r = 0; r < n; ++r) {
        fx_shard& s = out[r];
        s.tile_begin = T * r / n;
        s.tile_end = T * (r + 1) / n;
        s.z_lo = s.z_hi = s.own_lo = s.own_hi = 0;
        if (s.tile_end <= s.tile_begin) {  // more shards than tiles: an empty shard
            s.tile_end = s.tile_begin;
            continue;
        }
        const int64_t iz0 = s.tile_begin / per_row, iz1 = (s.tile_end - 1) / per_row;
        s.z_lo = zs[static_cast<size_t>(iz0)];
        s.z_hi = std::min<int64_t>(zs[static_cast<size_t>(iz1)] + patch, dz);
        s.own_lo = prev_live < 0 ? 0 : s.z_lo;
        if (prev_live >= 0) out[prev_live].own_hi = s.z_lo;
        s.own_hi = dz;
        prev_live = r;
    }
    return out;
}
}  // namespace fxh

namespace {

// Host barrier of the GPU threads (every thread arrives, also after a failure).
class Barrier {
  public:
    explicit Barrier(int n) : n_(n) {}
    void wait() {
        std::unique_lock<std::mutex> lk(m_);
        const int gen = gen_;
        if (++count_ == n_) {
            count_ = 0;
            ++gen_;
            cv_.notify_all();
            return;
        }
        cv_.wait(lk, [&] { return gen != gen_; });
    }

  private:
    std::mutex m_;
    std::condition_variable cv_;
    int n_, count_ = 0, gen_ = 0;
};

struct Exchange {
    int src, dst;
    int64_t z0, z1;
};

std::vector<Exchange> exchanges(const std::vector<fx_shard>& plan) {
    std::vector<Exchange> ex;
    for (int a = 0; a < static_cast<int>(plan.size()); ++a)
        for (int b = 0; b < static_cast<int>(plan.size()); ++b) {
            if (a == b || plan[a].tile_end <= plan[a].tile_begin || plan[b].tile_end <= plan[b].tile_begin) continue;
            const int64_t z0 = std::max(plan[a].z_lo, plan[b].own_lo), z1 = std::min(plan[a].z_hi, plan[b].own_hi);
            if (z1 > z0) ex.push_back({a, b, z0, z1});
        }
    return ex;
}

}  // namespace

extern "C" {

fx_status fx_ipc_buffer_alloc(int device, uint64_t bytes, void** dev_ptr, void* handle) {
    if (!dev_ptr || !handle || bytes == 0) return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_ipc_buffer_alloc: bad argument");
    *dev_ptr = nullptr;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMalloc(dev_ptr, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, *dev_ptr);
    if (e != cudaSuccess) {
        if (*dev_ptr) cudaFree(*dev_ptr);
        *dev_ptr = nullptr;
        return fxh::abi_error(FX_INTERNAL, std::string("fx_ipc_buffer_alloc: ") + cudaGetErrorString(e));
    }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(handle, &h, sizeof h);
    return FX_OK;
}

fx_status fx_ipc_buffer_free(int device, void* dev_ptr) {
    if (!dev_ptr) return FX_OK;
    cudaSetDevice(device);
    const cudaError_t e = cudaFree(dev_ptr);
    return e == cudaSuccess ? FX_OK : fxh::abi_error(FX_INTERNAL, std::string("fx_ipc_buffer_free: ") + cudaGetErrorString(e));
}

fx_status fx_ipc_open(int device, const void* handle, void** dev_ptr) {
    if (!handle || !dev_ptr) return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? FX_OK : fxh::abi_error(FX_INTERNAL, std::string("fx_ipc_open: ") + cudaGetErrorString(e));
}

fx_status fx_ipc_close(int device, void* dev_ptr) {
    if (!dev_ptr) return FX_OK;
    cudaSetDevice(device);
    const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    return e == cudaSuccess ? FX_OK : fxh::abi_error(FX_INTERNAL, std::string("fx_ipc_close: ") + cudaGetErrorString(e));
}

int fx_shard_plan(int64_t dz, int64_t dy, int64_t dx, int patch, double overlap, int nshards, fx_shard* out) {
    if (dz < 1 || dy < 1 || dx < 1 || patch < 1 || nshards < 1 || !(overlap >= 0.0 && overlap < 1.0)) return 0;
    const auto p = fxh::shard_plan(dz, dy, dx, patch, overlap, nshards);
    if (out) std::copy(p.begin(), p.end(), out);
    return nshards;
}

fx_status fx_predict_volume_multi(fx_net* const* nets, int n, const uint8_t* host_vol, int64_t dz, int64_t dy,
                                  int64_t dx, const fx_infer_opts* o, float* host_prob, uint8_t* host_u8) {
    try {
        if (!nets || n < 1 || !host_vol || !o) return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_predict_volume_multi: null argument");
        if (dz < 1 || dy < 1 || dx < 1) return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_predict_volume_multi: empty volume");
        if (o->patch % 64 != 0) return fxh::abi_error(FX_INVALID_ARGUMENT, "patch must be divisible by 64");
        if (o->tile[0] || o->tile[1] || o->tile[2])  // z-slab sharding plans cubic tiles
            return fxh::abi_error(FX_UNSUPPORTED, "fx_predict_volume_multi: cubic tiles only (opts.tile must be 0)");
        for (int i = 0; i < n; ++i) {
            if (!nets[i]) return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_predict_volume_multi: null net");
            if (nets[i]->net.patch() != o->patch)
                return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_predict_volume_multi: patch differs from a net's");
            for (int j = 0; j < i; ++j)
                if (nets[j] == nets[i]) return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_predict_volume_multi: a net twice");
        }
        if (n == 1) return fx_predict_volume(nets[0], host_vol, dz, dy, dx, o, host_prob, host_u8);
        const fxh::RunOpts ro = fxh::run_opts(o);
        if (ro.core_org[0] || ro.core_org[1] || ro.core_org[2] || ro.core_ext[0] > 0 || ro.core_ext[1] > 0 ||
            ro.core_ext[2] > 0)
            return fxh::abi_error(FX_UNSUPPORTED, "fx_predict_volume_multi: output crops are taken by fx_predict_volume only");
        const auto plan = fxh::shard_plan(dz, dy, dx, o->patch, o->overlap, n);
        const auto ex = exchanges(plan);
        // peer access between every pair of devices that can reach each other (NVLink / NVSwitch)
        std::vector<std::vector<int>> peer(n, std::vector<int>(n, 0));
        for (int i = 0; i < n; ++i)
            for (int j = 0; j < n; ++j) {
                if (i == j) continue;
                const int di = nets[i]->net.device(), dj = nets[j]->net.device();
                if (di == dj) {  // shards sharing a device read each other's accumulators directly
                    peer[i][j] = 1;
                    continue;
                }
                int can = 0;
                cudaDeviceCanAccessPeer(&can, di, dj);
                if (can) {
                    cudaSetDevice(di);
                    const cudaError_t e = cudaDeviceEnablePeerAccess(dj, 0);
                    if (e == cudaSuccess || e == cudaErrorPeerAccessAlreadyEnabled) peer[i][j] = 1;
                    cudaGetLastError();  // clear an already-enabled status
                }
            }
        const int P = o->patch;
        const auto g = fenix::ml::gaussian1d(P);
        const auto zs = fenix::ml::tile_starts(dz, P, o->overlap), ys = fenix::ml::tile_starts(dy, P, o->overlap),
                   xs = fenix::ml::tile_starts(dx, P, o->overlap);
        std::vector<float> wprof(static_cast<size_t>(dz + dy + dx));
        {
            const auto Wz = fenix::ml::weight_profile(g, zs, 0, dz, dz, P), Wy = fenix::ml::weight_profile(g, ys, 0, dy, dy, P),
                       Wx = fenix::ml::weight_profile(g, xs, 0, dx, dx, P);
            std::copy(Wz.begin(), Wz.end(), wprof.begin());
            std::copy(Wy.begin(), Wy.end(), wprof.begin() + dz);
            std::copy(Wx.begin(), Wx.end(), wprof.begin() + dz + dy);
        }
        const int64_t plane = dy * dx;
        std::vector<float*> accs(n, nullptr);
        std::vector<fxh::Status> st(n);
        std::atomic<bool> failed{false};
        Barrier bar(n);
        auto work = [&](int r) {
            fxh::Net& net = nets[r]->net;
            const fx_shard& p = plan[r];
            const bool live = p.tile_end > p.tile_begin;
            cudaSetDevice(net.device());
            cudaStream_t s = net.stream();
            float *d_w = nullptr, *d_tmp = nullptr;
            uint8_t *d_vol = nullptr, *d_out = nullptr;
            const int64_t nz = p.z_hi - p.z_lo, nown = p.own_hi - p.own_lo;
            auto run = [&](fxh::Status& out) {
                if (!live) return;
                // workspace: input slab, accumulator window, owned-plane outputs (f32 and/or u8)
                const size_t out_bytes = static_cast<size_t>(nown * plane) * ((host_prob ? 4 : 0) + (host_u8 ? 1 : 0));
                if ((out = net.workspace(static_cast<size_t>(nz * plane), static_cast<size_t>(nz * plane) * 4,
                                         std::max<size_t>(out_bytes, 16), &d_vol, &accs[r], &d_out))
                        .code)
                    return;
                cudaMemcpyAsync(d_vol, host_vol + p.z_lo * plane, static_cast<size_t>(nz * plane), cudaMemcpyHostToDevice, s);
                cudaMemsetAsync(accs[r], 0, static_cast<size_t>(nz * plane) * 4, s);
                if ((out = net.predict_tiles(d_vol, nz, dy, dx, p.z_lo, dz, fxk::TileDims{P, P, P}, o->overlap, o->channel, o->sigmoid,
                                             o->batch, p.tile_begin, p.tile_end, accs[r], s, 0, -1, o->tta, ro))
                        .code)
                    return;
                out = net.take_device_status();  // synchronises the stream: this GPU's blend is complete
            };
            try {
                run(st[r]);
            } catch (const std::exception& e) {
                st[r] = fxh::fail(FX_INTERNAL, std::string("internal error: ") + e.what());
            }
            if (!st[r].ok()) failed = true;
            bar.wait();  // every GPU's tiles are blended (or some GPU failed)
            if (!failed && live) try {
                fxh::Status& out = st[r];
                // fold in the bands other GPUs accumulated for the planes this GPU owns
                for (const Exchange& e : ex) {
                    if (e.dst != r || !out.ok()) continue;
                    const int64_t cnt = (e.z1 - e.z0) * plane;
                    float* dst = accs[r] + (e.z0 - p.z_lo) * plane;
                    const float* src = accs[e.src] + (e.z0 - plan[e.src].z_lo) * plane;
                    cudaError_t ce;
                    if (peer[r][e.src]) {  // the add kernel reads the neighbour's HBM over NVLink
                        ce = fxk::launch_accum_add(dst, src, cnt, s);
                    } else {  // no peer mapping: stage the band in this GPU's memory first
                        if (!d_tmp && cudaMalloc(&d_tmp, static_cast<size_t>(cnt) * 4) != cudaSuccess) {
                            out = fxh::fail(FX_INTERNAL, "cudaMalloc: band staging");
                            break;
                        }
                        ce = cudaMemcpyPeerAsync(d_tmp, net.device(), src, nets[e.src]->net.device(),
                                                 static_cast<size_t>(cnt) * 4, s);
                        if (ce == cudaSuccess) ce = fxk::launch_accum_add(dst, d_tmp, cnt, s);
                        if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
                        cudaFree(d_tmp);
                        d_tmp = nullptr;
                    }
                    if (ce != cudaSuccess) out = fxh::cuda_status(ce, "band fold");
                }
                if (out.ok() && nown > 0) {
                    if (cudaMalloc(&d_w, sizeof(float) * wprof.size()) != cudaSuccess) {
                        out = fxh::fail(FX_INTERNAL, "cudaMalloc: weight profiles");
                    } else {
                        cudaMemcpyAsync(d_w, wprof.data(), sizeof(float) * wprof.size(), cudaMemcpyHostToDevice, s);
                        float* d_prob = host_prob ? reinterpret_cast<float*>(d_out) : nullptr;
                        uint8_t* d_u8 = host_u8 ? d_out + (host_prob ? static_cast<size_t>(nown * plane) * 4 : 0) : nullptr;
                        // the accumulator window starts at plane z_lo, so does the Wz it is normalised by
                        cudaError_t ce = fxk::launch_accum_finalize(accs[r], nz, dy, dx, p.own_lo - p.z_lo, p.own_hi - p.z_lo,
                                                                    d_w + p.z_lo, d_w + dz, d_w + dz + dy, d_prob, d_u8, s);
                        if (ce == cudaSuccess && host_prob)
                            ce = cudaMemcpyAsync(host_prob + p.own_lo * plane, d_prob, static_cast<size_t>(nown * plane) * 4,
                                                 cudaMemcpyDeviceToHost, s);
                        if (ce == cudaSuccess && host_u8)
                            ce = cudaMemcpyAsync(host_u8 + p.own_lo * plane, d_u8, static_cast<size_t>(nown * plane),
                                                 cudaMemcpyDeviceToHost, s);
                        const cudaError_t cs = cudaStreamSynchronize(s);
                        if (ce == cudaSuccess) ce = cs;
                        if (ce != cudaSuccess) out = fxh::cuda_status(ce, "finalise");
                    }
                }
                if (!out.ok()) failed = true;
            } catch (const std::exception& e) {
                st[r] = fxh::fail(FX_INTERNAL, std::string("internal error: ") + e.what());
                failed = true;
            }
            bar.wait();  // no GPU reads a neighbour's accumulator after this point
            if (d_w) cudaFree(d_w);
        };
        std::vector<std::thread> th;
        for (int r = 1; r < n; ++r) th.emplace_back(work, r);
        work(0);
        for (auto& t : th) t.join();
        for (int r = 0; r < n; ++r)
            if (!st[r].ok()) return fxh::abi_error(st[r].code, "GPU " + std::to_string(r) + ": " + st[r].msg);
        return FX_OK;
    } catch (...) {
        return fxh::abi_exception();
    }
}

}  // extern "C"
