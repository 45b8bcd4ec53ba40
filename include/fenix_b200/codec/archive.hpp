// fenix_b200/codec/archive.hpp — header-only C++ side of the .fxvol entry points, mirroring the
// reference's codec::VolumeArchive (src/codec/archive.hpp:132-1217) for the calls the
// surface-prediction path makes (src/ml/inference.cpp:553-567 input, 333-355 output): open /
// create, dims / params / nlods / src_dtype, coverage, chunk payloads, read_volume_as<u8>(0),
// write_volume<u8>, close. Chunk decode and encode run on the GPU (`device`); the file layout and
// the tile bitstream are the reference's.
#pragma once

#include "fenix_b200/ml/infer.hpp"

#include <span>
#include <string>
#include <utility>

namespace fenix_b200::codec {

enum class Coverage : u8 { Absent = 0, Zero = 1, Real = 2 };
enum class DType : u8 { u8 = 0, u16, u32, s8, s16, s32, f16, f32 };

// The DctParams fields an archive stores (archive.hpp:236-238); the rest keep their defaults.
struct DctParams {
    f32 q = 8.0f;
    f32 hf_exp = 0.65f;
    f32 dz_frac = 0.80f;
};

class VolumeArchive {
public:
    VolumeArchive() = default;
    VolumeArchive(const VolumeArchive&) = delete;
    VolumeArchive& operator=(const VolumeArchive&) = delete;
    VolumeArchive(VolumeArchive&& o) noexcept : h_(std::exchange(o.h_, nullptr)), device_(o.device_) {}
    VolumeArchive& operator=(VolumeArchive&& o) noexcept {
        if (this != &o) {
            release();
            h_ = std::exchange(o.h_, nullptr);
            device_ = o.device_;
        }
        return *this;
    }
    ~VolumeArchive() { release(); }

    [[nodiscard]] static Expected<VolumeArchive> create(const std::string& path, Extent3 dims, DctParams bp,
                                                        DType src_dtype = DType::u8, int device = 0) {
        VolumeArchive a;
        a.device_ = device;
        const fx_status st = fx_fxvol_create(path.c_str(), dims.z, dims.y, dims.x, bp.q,
                                             static_cast<int32_t>(src_dtype), &a.h_);
        if (st != FX_OK) return err_status(st, "VolumeArchive::create(" + path + ")");
        return a;
    }
    [[nodiscard]] static Expected<VolumeArchive> open(const std::string& path, int device = 0) {
        VolumeArchive a;
        a.device_ = device;
        const fx_status st = fx_fxvol_open(path.c_str(), &a.h_);
        if (st != FX_OK) return err_status(st, "VolumeArchive::open(" + path + ")");
        return a;
    }

    [[nodiscard]] Extent3 dims() const {
        const fx_fxvol_info i = info();
        return {i.dims[0], i.dims[1], i.dims[2]};
    }
    [[nodiscard]] DctParams params() const {
        const fx_fxvol_info i = info();
        return {i.q, i.hf_exp, i.dz_frac};
    }
    [[nodiscard]] uint32_t nlods() const { return info().nlods; }
    [[nodiscard]] DType src_dtype() const { return static_cast<DType>(info().src_dtype); }

    [[nodiscard]] Coverage coverage(s64 lod, ChunkCoord c) const {
        int cov = 0;
        const u8* p = nullptr;
        uint64_t n = 0;
        if (fx_fxvol_chunk_payload(h_, static_cast<int>(lod), c.z, c.y, c.x, &cov, &p, &n) != FX_OK)
            return Coverage::Absent;
        return static_cast<Coverage>(cov);
    }
    // A REAL chunk's crc-checked payload (empty for ABSENT / ZERO), valid until close().
    [[nodiscard]] Expected<std::span<const u8>> chunk_payload(s64 lod, ChunkCoord c) const {
        int cov = 0;
        const u8* p = nullptr;
        uint64_t n = 0;
        const fx_status st = fx_fxvol_chunk_payload(h_, static_cast<int>(lod), c.z, c.y, c.x, &cov, &p, &n);
        if (st != FX_OK) return err_status(st, "VolumeArchive::chunk_payload");
        return std::span<const u8>(p, static_cast<std::size_t>(n));
    }
    // write_chunk_payload (archive.hpp:350-362); an empty payload records a ZERO chunk.
    [[nodiscard]] Expected<void> write_chunk_payload(s64 lod, ChunkCoord c, std::span<const u8> payload) {
        const fx_status st =
            fx_fxvol_write_chunk_payload(h_, static_cast<int>(lod), c.z, c.y, c.x, payload.data(), payload.size());
        if (st != FX_OK) return err_status(st, "VolumeArchive::write_chunk_payload");
        return {};
    }
    [[nodiscard]] Expected<void> set_nlods(uint32_t n) {
        const fx_status st = fx_fxvol_set_nlods(h_, n);
        if (st != FX_OK) return err_status(st, "VolumeArchive::set_nlods");
        return {};
    }
    // read_volume_as<u8>(0) (archive.hpp:550-590): LOD 0, decoded on the device.
    [[nodiscard]] Expected<Volume<u8>> read_volume_u8() const {
        Volume<u8> out(dims());
        const fx_status st = fx_fxvol_read_volume_u8(h_, device_, out.data());
        if (st != FX_OK) return err_status(st, "VolumeArchive::read_volume_as<u8>");
        return out;
    }
    // write_volume<u8> (archive.hpp:418-440): LOD 0 and the octave pyramid, encoded on the device.
    [[nodiscard]] Expected<void> write_volume(VolumeView<const u8> vol) {
        if (!(vol.dims() == dims())) return err(Errc::invalid_argument, "VolumeArchive::write_volume: dims mismatch");
        std::vector<u8> tmp;
        const u8* src = ml::detail::contiguous_input(vol, tmp);
        const fx_status st = fx_fxvol_write_volume_u8(h_, src, device_);
        if (st != FX_OK) return err_status(st, "VolumeArchive::write_volume");
        return {};
    }
    // close(): commit + trim for writers (archive.hpp:867-894).
    [[nodiscard]] Expected<void> close() {
        const fx_status st = fx_fxvol_close(std::exchange(h_, nullptr));
        if (st != FX_OK) return err_status(st, "VolumeArchive::close");
        return {};
    }

private:
    fx_fxvol_info info() const {
        fx_fxvol_info i{};
        fx_fxvol_get_info(h_, &i);
        return i;
    }
    void release() {
        if (h_) fx_fxvol_close(std::exchange(h_, nullptr));
    }
    fx_fxvol* h_ = nullptr;
    int device_ = 0;
};

}  // namespace fenix_b200::codec

namespace fenix_b200::ml {

// predict-surface over archives: the u8 .fxvol input decoded on the net's device, the prediction
// written as a u8 .fxvol at q (inference.cpp:333-356; the reference's default q = 32), the volume
// resident on the device from decode to encode.
[[nodiscard]] inline Expected<void> predict_surface_fxvol(B200Net& net, const std::string& in_path,
                                                          const std::string& out_path, const InferOptions& opt,
                                                          float q = 32.0f) {
    auto o = to_fx(opt);
    if (!o) return std::unexpected(o.error());
    if (o->batch > net.batch()) o->batch = net.batch();
    const fx_status st = fx_predict_fxvol(net.handle(), in_path.c_str(), out_path.c_str(), &*o, q);
    if (st != FX_OK) return err_status(st, "predict_surface_fxvol");
    return {};
}

}  // namespace fenix_b200::ml
