// fxvol_api.cu — the .fxvol entry points of include/fenix_b200.h: the archive container
// (src/codec/archive.hpp VolumeArchive) with LOD-0 reads decoded and writes encoded on the device,
// the tile codec over host buffers (src/codec/dct_block.hpp encode_tile_dct / decode_tile_dct),
// and the predict-surface command over archives (src/ml/inference.cpp:540-567 input, 333-355
// output) with the volume resident on the device from decode to encode.
#include "fenix_b200.h"
#include "fxvol.cuh"
#include "fxvol_archive.hpp"
#include "net.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

namespace fxh {
fx_status abi_error(int code, const std::string& msg);
fx_status abi_exception();
}  // namespace fxh

struct fx_fxvol {
    fxh::FxvolArchive a;
};

namespace {

using fxh::abi_error;

constexpr int64_t kChunk = 64;
constexpr size_t kDecodeBatchBytes = 256u << 20;  // payload bytes staged per decode call

fx_status cuda_err(cudaError_t e, const char* what) {
    return abi_error(FX_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
}

fx_status codec_err(const fxh::CodecStatus& c) {
    return abi_error(c.code == 5 ? FX_DECODE_ERROR : FX_INTERNAL, c.msg);
}

// per-device codec objects (scratch kept between calls)
fxh::FxvCodec& codec_for(int device) {
    static std::unique_ptr<fxh::FxvCodec> codecs[64];
    auto& c = codecs[device & 63];
    if (!c) c = std::make_unique<fxh::FxvCodec>();
    return *c;
}

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    bool alloc(size_t n) {
        return cudaMalloc(&p, n ? n : 1) == cudaSuccess;
    }
};

struct HostPinned {
    void* p = nullptr;
    ~HostPinned() {
        if (p) cudaFreeHost(p);
    }
    bool alloc(size_t n) { return cudaMallocHost(&p, n ? n : 1) == cudaSuccess; }
};

// 2x box downsample of one octave (archive.hpp:914-938): the mean of the in-bounds voxels of each
// 2^3 cell, summed in (dz, dy, dx) order in f32.
template <bool U8>
__global__ void fxv_downsample2(const uint8_t* __restrict__ in8, const float* __restrict__ in32, int64_t dz, int64_t dy,
                                int64_t dx, float* __restrict__ out, int64_t oz, int64_t oy, int64_t ox) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= oz * oy * ox) return;
    const int64_t x = i % ox, y = (i / ox) % oy, z = i / (ox * oy);
    float sum = 0.0f;
    int n = 0;
    for (int a = 0; a < 2; ++a)
        for (int b = 0; b < 2; ++b)
            for (int c = 0; c < 2; ++c) {
                const int64_t sz = 2 * z + a, sy = 2 * y + b, sx = 2 * x + c;
                if (sz < dz && sy < dy && sx < dx) {
                    const int64_t k = (sz * dy + sy) * dx + sx;
                    sum = __fadd_rn(sum, U8 ? static_cast<float>(in8[k]) : in32[k]);
                    ++n;
                }
            }
    out[i] = n ? __fdiv_rn(sum, static_cast<float>(n)) : 0.0f;
}

// read_volume_as<u8>(0) (archive.hpp:550-590) into a device volume: REAL chunks decoded on the
// device, ABSENT / ZERO chunks left at the fill value 0.
fx_status decode_lod0(const fxh::FxvolArchive& a, int device, uint8_t* d_vol, cudaStream_t s) {
    const auto& m = a.meta();
    const int64_t dz = m.dims[0], dy = m.dims[1], dx = m.dims[2];
    cudaError_t e = cudaMemsetAsync(d_vol, 0, static_cast<size_t>(dz) * dy * dx, s);
    if (e != cudaSuccess) return cuda_err(e, "cudaMemsetAsync");
    const int64_t cz = (dz + kChunk - 1) / kChunk, cy = (dy + kChunk - 1) / kChunk, cx = (dx + kChunk - 1) / kChunk;
    const fxk::FxvParams p = fxk::fxv_make_params(m.q, m.hf_exp, m.dz_frac);
    fxh::FxvCodec& codec = codec_for(device);
    HostPinned stage;
    DevBuf blob;
    size_t stage_cap = 0;
    std::vector<fxk::FxvDecTile> tiles;
    std::vector<std::pair<const uint8_t*, uint64_t>> spans;
    auto flush = [&]() -> fx_status {
        if (tiles.empty()) return FX_OK;
        uint64_t total = 0;
        for (auto& sp : spans) total += sp.second;
        if (total > stage_cap) {
            if (stage.p) cudaFreeHost(stage.p);
            if (blob.p) cudaFree(blob.p);
            stage.p = blob.p = nullptr;
            if (!stage.alloc(total) || !blob.alloc(total)) return abi_error(FX_INTERNAL, "fxvol: staging allocation");
            stage_cap = total;
        }
        uint64_t o = 0;
        for (size_t k = 0; k < spans.size(); ++k) {
            std::memcpy(static_cast<uint8_t*>(stage.p) + o, spans[k].first, spans[k].second);
            tiles[k].off = o;
            o += spans[k].second;
        }
        cudaMemcpyAsync(blob.p, stage.p, total, cudaMemcpyHostToDevice, s);
        const fxh::CodecStatus cs = codec.decode(static_cast<const uint8_t*>(blob.p), tiles.data(),
                                                 static_cast<int64_t>(tiles.size()), p, d_vol, dz, dy, dx, nullptr, s);
        if (cs.code) return codec_err(cs);
        tiles.clear();
        spans.clear();
        return FX_OK;
    };
    uint64_t pending = 0;
    for (int64_t z = 0; z < cz; ++z)
        for (int64_t y = 0; y < cy; ++y)
            for (int64_t x = 0; x < cx; ++x) {
                int cov = 0;
                const uint8_t* pl = nullptr;
                uint64_t len = 0;
                const std::string err = a.chunk(0, z, y, x, &cov, &pl, &len);
                if (!err.empty()) return abi_error(FX_DECODE_ERROR, err);
                if (cov != fxh::kReal) continue;
                if (len > 0xffffffffull) return abi_error(FX_DECODE_ERROR, "chunk payload too large");
                tiles.push_back(fxk::FxvDecTile{0, static_cast<uint32_t>(len), 0, z * kChunk, y * kChunk, x * kChunk});
                spans.emplace_back(pl, len);
                pending += len;
                if (pending >= kDecodeBatchBytes) {
                    if (fx_status r = flush()) return r;
                    pending = 0;
                }
            }
    return flush();
}

// Encode every chunk of one LOD level (write_level_, archive.hpp:942-994) and commit it in chunk
// order; an all-zero chunk becomes a ZERO slot.
fx_status encode_level(fxh::FxvolArchive& a, int lod, const uint8_t* d8, const float* d32, const int64_t d[3],
                       int device, cudaStream_t s) {
    const auto& m = a.meta();
    const int64_t cz = (d[0] + kChunk - 1) / kChunk, cy = (d[1] + kChunk - 1) / kChunk, cx = (d[2] + kChunk - 1) / kChunk;
    std::vector<fxk::FxvEncTile> tiles;
    tiles.reserve(static_cast<size_t>(cz * cy * cx));
    for (int64_t z = 0; z < cz; ++z)
        for (int64_t y = 0; y < cy; ++y)
            for (int64_t x = 0; x < cx; ++x) tiles.push_back(fxk::FxvEncTile{z * kChunk, y * kChunk, x * kChunk});
    fxk::FxvParams p = fxk::fxv_make_params(m.q, m.hf_exp, m.dz_frac);
    std::vector<uint8_t> pay;
    std::vector<uint64_t> off;
    std::vector<uint32_t> len;
    const fxh::CodecStatus cs = codec_for(device).encode(d8, d32, d[0], d[1], d[2], tiles.data(),
                                                         static_cast<int64_t>(tiles.size()), p, pay, off, len, s, true);
    if (cs.code) return codec_err(cs);
    for (size_t k = 0; k < tiles.size(); ++k) {
        const std::string err = a.put(lod, tiles[k].z0 / kChunk, tiles[k].y0 / kChunk, tiles[k].x0 / kChunk,
                                      pay.data() + off[k], len[k]);
        if (!err.empty()) return abi_error(FX_IO_ERROR, err);
    }
    return FX_OK;
}

// write_volume<u8> (archive.hpp:418-440): LOD 0 from the u8 volume, then the octave pyramid in f32.
fx_status encode_volume(fxh::FxvolArchive& a, const uint8_t* d_vol, int device, cudaStream_t s) {
    const auto& m = a.meta();
    int64_t d[3] = {m.dims[0], m.dims[1], m.dims[2]};
    if (fx_status r = encode_level(a, 0, d_vol, nullptr, d, device, s)) return r;
    auto fits = [](const int64_t* v) { return v[0] <= kChunk && v[1] <= kChunk && v[2] <= kChunk; };
    if (fits(d)) {
        a.set_nlods(1);
        return FX_OK;
    }
    DevBuf cur, nxt;
    int lod = 0;
    const uint8_t* src8 = d_vol;
    const float* src32 = nullptr;
    do {
        const int64_t o[3] = {(d[0] + 1) / 2, (d[1] + 1) / 2, (d[2] + 1) / 2};
        const int64_t no = o[0] * o[1] * o[2];
        if (!nxt.alloc(sizeof(float) * static_cast<size_t>(no))) return abi_error(FX_INTERNAL, "cudaMalloc: pyramid level");
        const unsigned g = static_cast<unsigned>((no + 255) / 256);
        if (src8)
            fxv_downsample2<true><<<g, 256, 0, s>>>(src8, nullptr, d[0], d[1], d[2], static_cast<float*>(nxt.p), o[0],
                                                   o[1], o[2]);
        else
            fxv_downsample2<false><<<g, 256, 0, s>>>(nullptr, src32, d[0], d[1], d[2], static_cast<float*>(nxt.p),
                                                    o[0], o[1], o[2]);
        if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) return cuda_err(e, "fxv_downsample2");
        std::swap(cur.p, nxt.p);
        if (nxt.p) {
            cudaStreamSynchronize(s);
            cudaFree(nxt.p);
            nxt.p = nullptr;
        }
        src8 = nullptr;
        src32 = static_cast<const float*>(cur.p);
        for (int k = 0; k < 3; ++k) d[k] = o[k];
        ++lod;
        if (fx_status r = encode_level(a, lod, nullptr, src32, d, device, s)) return r;
    } while (!fits(d) && lod + 1 < 20);
    a.set_nlods(static_cast<uint32_t>(lod + 1));
    return FX_OK;
}

template <class F>
fx_status guarded(F&& f) {
    try {
        return f();
    } catch (...) {
        return fxh::abi_exception();
    }
}

}  // namespace

extern "C" {

fx_status fx_fxvol_open(const char* path, fx_fxvol** out) {
    return guarded([&]() -> fx_status {
        if (!path || !out) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_open: null argument");
        *out = nullptr;
        auto h = std::make_unique<fx_fxvol>();
        const std::string err = h->a.open(path);
        if (!err.empty())
            return abi_error(err.rfind("cannot open", 0) == 0 ? FX_NOT_FOUND : FX_DECODE_ERROR, err);
        *out = h.release();
        return FX_OK;
    });
}

fx_status fx_fxvol_create(const char* path, int64_t dz, int64_t dy, int64_t dx, float q, int32_t src_dtype,
                          fx_fxvol** out) {
    return guarded([&]() -> fx_status {
        if (!path || !out) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_create: null argument");
        *out = nullptr;
        auto h = std::make_unique<fx_fxvol>();
        const int64_t d[3] = {dz, dy, dx};
        const std::string err = h->a.create(path, d, q, 0.65f, 0.80f, static_cast<uint32_t>(src_dtype));
        if (!err.empty()) return abi_error(err.rfind("cannot", 0) == 0 ? FX_IO_ERROR : FX_INVALID_ARGUMENT, err);
        *out = h.release();
        return FX_OK;
    });
}

fx_status fx_fxvol_get_info(const fx_fxvol* h, fx_fxvol_info* out) {
    if (!h || !out) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_get_info: null argument");
    const auto& m = h->a.meta();
    for (int k = 0; k < 3; ++k) out->dims[k] = m.dims[k];
    out->q = m.q;
    out->hf_exp = m.hf_exp;
    out->dz_frac = m.dz_frac;
    out->nlods = m.nlods;
    out->src_dtype = static_cast<int32_t>(m.dtype);
    out->sealed = m.data_off != 0;
    return FX_OK;
}

fx_status fx_fxvol_chunk_payload(const fx_fxvol* h, int lod, int64_t cz, int64_t cy, int64_t cx, int* coverage,
                                 const uint8_t** payload, uint64_t* len) {
    if (!h || !coverage || !payload || !len) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_chunk_payload: null argument");
    const std::string err = h->a.chunk(lod, cz, cy, cx, coverage, payload, len);
    return err.empty() ? FX_OK : abi_error(FX_DECODE_ERROR, err);
}

fx_status fx_fxvol_write_chunk_payload(fx_fxvol* h, int lod, int64_t cz, int64_t cy, int64_t cx,
                                       const uint8_t* payload, uint64_t len) {
    if (!h || (len && !payload)) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_write_chunk_payload: null argument");
    const std::string err = h->a.put(lod, cz, cy, cx, payload, len);
    return err.empty() ? FX_OK : abi_error(FX_INVALID_ARGUMENT, err);
}

fx_status fx_fxvol_set_nlods(fx_fxvol* h, uint32_t nlods) {
    if (!h || nlods < 1 || nlods > 20) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_set_nlods: bad argument");
    h->a.set_nlods(nlods);
    return FX_OK;
}

fx_status fx_fxvol_close(fx_fxvol* h) {
    if (!h) return FX_OK;
    const std::string err = h->a.close();
    delete h;
    return err.empty() ? FX_OK : abi_error(FX_IO_ERROR, err);
}

fx_status fx_fxvol_read_volume_u8(const fx_fxvol* h, int device, uint8_t* host_out) {
    return guarded([&]() -> fx_status {
        if (!h || !host_out) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_read_volume_u8: null argument");
        const auto& m = h->a.meta();
        if (m.dtype != 0) return abi_error(FX_UNSUPPORTED, "fx_fxvol_read_volume_u8: not a u8 archive");
        if (cudaError_t e = cudaSetDevice(device); e != cudaSuccess) return cuda_err(e, "cudaSetDevice");
        const size_t nv = static_cast<size_t>(m.dims[0]) * m.dims[1] * m.dims[2];
        cudaStream_t s = nullptr;
        cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        DevBuf vol;
        fx_status r = vol.alloc(nv) ? decode_lod0(h->a, device, static_cast<uint8_t*>(vol.p), s)
                                    : abi_error(FX_INTERNAL, "cudaMalloc: volume");
        if (!r) {
            cudaMemcpyAsync(host_out, vol.p, nv, cudaMemcpyDeviceToHost, s);
            if (cudaError_t e = cudaStreamSynchronize(s); e != cudaSuccess) r = cuda_err(e, "fxvol read");
        }
        cudaStreamDestroy(s);
        return r;
    });
}

fx_status fx_fxvol_write_volume_u8(fx_fxvol* h, const uint8_t* host_vol, int device) {
    return guarded([&]() -> fx_status {
        if (!h || !host_vol) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_write_volume_u8: null argument");
        if (!h->a.writable()) return abi_error(FX_IO_ERROR, "archive opened read-only");
        const auto& m = h->a.meta();
        if (m.dtype != 0) return abi_error(FX_UNSUPPORTED, "fx_fxvol_write_volume_u8: not a u8 archive");
        if (cudaError_t e = cudaSetDevice(device); e != cudaSuccess) return cuda_err(e, "cudaSetDevice");
        const size_t nv = static_cast<size_t>(m.dims[0]) * m.dims[1] * m.dims[2];
        cudaStream_t s = nullptr;
        cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        DevBuf vol;
        fx_status r = FX_OK;
        if (!vol.alloc(nv)) r = abi_error(FX_INTERNAL, "cudaMalloc: volume");
        if (!r) {
            cudaMemcpyAsync(vol.p, host_vol, nv, cudaMemcpyHostToDevice, s);
            r = encode_volume(h->a, static_cast<const uint8_t*>(vol.p), device, s);
        }
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
        return r;
    });
}

fx_status fx_fxvol_decode_tiles(const uint8_t* payloads, uint64_t payload_bytes, const uint64_t* offsets,
                                const uint32_t* lengths, int64_t n, float q, float hf_exp, float dz_frac, int device,
                                uint8_t* out_u8, float* out_f32) {
    return guarded([&]() -> fx_status {
        if (n < 0 || (n && (!payloads || !offsets || !lengths)) || (!out_u8 && !out_f32))
            return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_decode_tiles: bad argument");
        if (!(q > 0.0f)) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_decode_tiles: bad quant step");
        for (int64_t k = 0; k < n; ++k)
            if (offsets[k] > payload_bytes || lengths[k] > payload_bytes - offsets[k])
                return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_decode_tiles: payload span outside the buffer");
        if (n == 0) return FX_OK;
        if (cudaError_t e = cudaSetDevice(device); e != cudaSuccess) return cuda_err(e, "cudaSetDevice");
        cudaStream_t s = nullptr;
        cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        const size_t tv = static_cast<size_t>(kChunk * kChunk * kChunk);
        DevBuf blob, u8, f32;
        fx_status r = FX_OK;
        if (!blob.alloc(payload_bytes) || !u8.alloc(tv * n) || (out_f32 && !f32.alloc(sizeof(float) * tv * n)))
            r = abi_error(FX_INTERNAL, "cudaMalloc: decode buffers");
        if (!r) {
            cudaMemcpyAsync(blob.p, payloads, payload_bytes, cudaMemcpyHostToDevice, s);
            cudaMemsetAsync(u8.p, 0, tv * n, s);
            std::vector<fxk::FxvDecTile> tiles(static_cast<size_t>(n));
            for (int64_t k = 0; k < n; ++k) tiles[k] = fxk::FxvDecTile{offsets[k], lengths[k], 0, k * kChunk, 0, 0};
            const fxk::FxvParams p = fxk::fxv_make_params(q, hf_exp, dz_frac);
            const fxh::CodecStatus cs =
                codec_for(device).decode(static_cast<const uint8_t*>(blob.p), tiles.data(), n, p, static_cast<uint8_t*>(u8.p),
                                         n * kChunk, kChunk, kChunk, static_cast<float*>(f32.p), s);
            if (cs.code) r = codec_err(cs);
        }
        if (!r && out_u8) cudaMemcpyAsync(out_u8, u8.p, tv * n, cudaMemcpyDeviceToHost, s);
        if (!r && out_f32) cudaMemcpyAsync(out_f32, f32.p, sizeof(float) * tv * n, cudaMemcpyDeviceToHost, s);
        if (cudaError_t e = cudaStreamSynchronize(s); !r && e != cudaSuccess) r = cuda_err(e, "fxvol decode");
        cudaStreamDestroy(s);
        return r;
    });
}

fx_status fx_fxvol_encode_tiles(const uint8_t* tiles_u8, const float* tiles_f32, int64_t n, float q, float hf_exp,
                                float dz_frac, int device, uint8_t* out, uint64_t cap, uint64_t* offsets,
                                uint32_t* lengths) {
    return guarded([&]() -> fx_status {
        if (n < 0 || (n && (!tiles_u8 == !tiles_f32)) || (n && (!offsets || !lengths)))
            return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_encode_tiles: bad argument");
        if (!(q > 0.0f)) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_encode_tiles: bad quant step");
        if (n == 0) return FX_OK;
        if (cudaError_t e = cudaSetDevice(device); e != cudaSuccess) return cuda_err(e, "cudaSetDevice");
        cudaStream_t s = nullptr;
        cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        const size_t tv = static_cast<size_t>(kChunk * kChunk * kChunk);
        const size_t bytes = tv * n * (tiles_u8 ? 1 : sizeof(float));
        DevBuf src;
        fx_status r = src.alloc(bytes) ? FX_OK : abi_error(FX_INTERNAL, "cudaMalloc: tiles");
        std::vector<uint8_t> pay;
        std::vector<uint64_t> off;
        std::vector<uint32_t> len;
        if (!r) {
            cudaMemcpyAsync(src.p, tiles_u8 ? static_cast<const void*>(tiles_u8) : tiles_f32, bytes,
                            cudaMemcpyHostToDevice, s);
            std::vector<fxk::FxvEncTile> tiles(static_cast<size_t>(n));
            for (int64_t k = 0; k < n; ++k) tiles[k] = fxk::FxvEncTile{k * kChunk, 0, 0};
            const fxk::FxvParams p = fxk::fxv_make_params(q, hf_exp, dz_frac);
            const fxh::CodecStatus cs = codec_for(device).encode(
                tiles_u8 ? static_cast<const uint8_t*>(src.p) : nullptr, tiles_f32 ? static_cast<const float*>(src.p) : nullptr,
                n * kChunk, kChunk, kChunk, tiles.data(), n, p, pay, off, len, s, false);
            if (cs.code) r = codec_err(cs);
        }
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
        if (r) return r;
        uint64_t o = 0;
        for (int64_t k = 0; k < n; ++k) o += len[k];
        if (o > cap) return abi_error(FX_INVALID_ARGUMENT, "fx_fxvol_encode_tiles: output buffer too small (" +
                                                               std::to_string(o) + " bytes needed)");
        o = 0;
        for (int64_t k = 0; k < n; ++k) {
            std::memcpy(out + o, pay.data() + off[k], len[k]);
            offsets[k] = o;
            lengths[k] = len[k];
            o += len[k];
        }
        return FX_OK;
    });
}

fx_status fx_predict_fxvol(fx_net* net, const char* in_path, const char* out_path, const fx_infer_opts* o,
                           float out_q) {
    return guarded([&]() -> fx_status {
        if (!net || !in_path || !out_path || !o) return abi_error(FX_INVALID_ARGUMENT, "fx_predict_fxvol: null argument");
        if (o->patch % 64 != 0) return abi_error(FX_INVALID_ARGUMENT, "patch must be divisible by 64");
        if (o->tile[0] || o->tile[1] || o->tile[2])
            return abi_error(FX_UNSUPPORTED, "fx_predict_fxvol: cubic tiles only (opts.tile must be 0)");
        for (int a = 0; a < 3; ++a)
            if (o->core_org[a] || o->core_ext[a] > 0)
                return abi_error(FX_UNSUPPORTED, "fx_predict_fxvol: the prediction archive covers the whole input (no crop)");
        fxh::FxvolArchive in;
        if (std::string err = in.open(in_path); !err.empty())
            return abi_error(err.rfind("cannot open", 0) == 0 ? FX_NOT_FOUND : FX_DECODE_ERROR, err);
        const auto& m = in.meta();
        if (m.dtype != 0) return abi_error(FX_UNSUPPORTED, "fx_predict_fxvol: input archive is not u8");
        const int dev = net->net.device();
        cudaSetDevice(dev);
        cudaStream_t s = net->net.stream();
        const int64_t dz = m.dims[0], dy = m.dims[1], dx = m.dims[2];
        const size_t nv = static_cast<size_t>(dz) * dy * dx;
        uint8_t *d_vol = nullptr, *d_u8 = nullptr;
        float* d_acc = nullptr;
        fxh::Status st = net->net.workspace(nv, nv * sizeof(float), nv, &d_vol, &d_acc, &d_u8);
        if (!st.ok()) return abi_error(st.code, st.msg);
        if (fx_status r = decode_lod0(in, dev, d_vol, s)) return r;
        if (fx_status r = fxh::predict_resident(net, d_vol, dz, dy, dx, o, d_acc, nullptr, d_u8)) return r;
        // predictions are written u8-native at q = 32 unless overridden (inference.cpp:333-341)
        const float q = out_q > 0.0f ? out_q : 32.0f;
        fxh::FxvolArchive outa;
        const int64_t d[3] = {dz, dy, dx};
        if (std::string err = outa.create(out_path, d, q, 0.65f, 0.80f, 0); !err.empty())
            return abi_error(FX_IO_ERROR, err);
        if (fx_status r = encode_volume(outa, d_u8, dev, s)) return r;
        if (std::string err = outa.close(); !err.empty()) return abi_error(FX_IO_ERROR, err);
        return FX_OK;
    });
}

}  // extern "C"
