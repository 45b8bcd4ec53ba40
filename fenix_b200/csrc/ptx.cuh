// ptx.cuh — thin inline-PTX wrappers for the sm_100a features the kernels use: mbarriers,
// bulk (non-tensor) async copies, tcgen05 TMEM allocation / MMA / commit / load, and the
// matrix + instruction descriptors tcgen05.mma consumes. Every wait is bounded: a wait that
// runs out records an error code in a device status word and returns false, so a bug shows
// up as a host-visible status instead of a hung GPU.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "optype.cuh"

namespace fxk {

// ---- status word ---------------------------------------------------------------------------
// Device-side error codes written (first writer wins) into the caller-provided status word.
enum : uint32_t {
    kStatusOk = 0,
    kStatusTimeoutFull = 0x100,    // MMA issuer waited too long for a smem stage
    kStatusTimeoutEmpty = 0x200,   // producer waited too long for a free smem stage
    kStatusTimeoutAcc = 0x300,     // epilogue waited too long for an accumulator
    kStatusTimeoutAccFree = 0x400, // MMA issuer waited too long for a drained accumulator
    kStatusTimeoutDrain = 0x500,   // final drain of in-flight copies timed out
    kStatusTimeoutExchange = 0x600, // fold epilogue waited too long for the row exchange
    kStatusBadTmem = 0x700,        // TMEM allocation returned an address outside the columns asked for
};

__device__ __forceinline__ void set_status(uint32_t* st, uint32_t code) {
    if (st) atomicCAS(st, 0u, code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// One lane of the (converged) warp gets true: the issuing lane of warp-wide role loops, whose
// control flow and operands stay warp-uniform.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\telect.sync rx|px, %1;\n\tselp.u32 %0, 1, 0, px;\n\t}"
        : "=r"(pred)
        : "r"(0xffffffffu));
    return pred != 0;
}

// ---- mbarrier --------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on a phase parity. Gives up after `limit_ns` of wall time, or as soon as
// *abort is set by another role of the same CTA. Returns true when the phase completed.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const volatile int* abort,
                                          uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (abort && *abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) return false;
        }
    }
}

// ---- bulk async copy global -> shared (1-D, no tensor map) ----------------------------------
// dst/src 16-byte aligned, bytes a multiple of 16; completion is signalled as tx bytes on bar.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// ---- tcgen05 ----------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/f16 inputs, f32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Same with 8-bit float inputs (kind::f8f6f4, e4m3 x e4m3, f32 accumulate).
__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Predicated forms for warp-wide issue loops: every lane runs the (warp-uniform) code, only the
// lane with issue != 0 executes the tcgen05 instruction.
__device__ __forceinline__ void mma_f16_if(uint32_t issue, uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 q, %5, 0;\n\t"
        "@q tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(issue)
        : "memory");
}
__device__ __forceinline__ void mma_f8_if(uint32_t issue, uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 q, %5, 0;\n\t"
        "@q tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(issue)
        : "memory");
}
// Three MMAs sharing one A tile (the x-tap fold): the first reads A from shared memory into the
// A collector, the second reuses it, the third reuses and releases it; B and D differ.
#define FX_MMA3(KIND)                                                                                           \
    asm volatile(                                                                                               \
        "{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %6, 0;\n\tsetp.ne.b32 q, %7, 0;\n\t"                    \
        "@q tcgen05.mma.cta_group::1.kind::" KIND ".collector::a::fill [%0], %3, %4, %5, p;\n\t"              \
        "@q tcgen05.mma.cta_group::1.kind::" KIND ".collector::a::use [%1], %3, %8, %5, p;\n\t"               \
        "@q tcgen05.mma.cta_group::1.kind::" KIND ".collector::a::lastuse [%2], %3, %9, %5, p;\n\t}" ::"r"(d0), \
        "r"(d1), "r"(d2), "l"(a_desc), "l"(b0), "r"(idesc), "r"(accumulate), "r"(issue), "l"(b1), "l"(b2)     \
        : "memory")
__device__ __forceinline__ void mma3_f16_if(uint32_t issue, uint32_t d0, uint32_t d1, uint32_t d2, uint64_t a_desc,
                                            uint64_t b0, uint64_t b1, uint64_t b2, uint32_t idesc,
                                            uint32_t accumulate) {
    FX_MMA3("f16");
}
__device__ __forceinline__ void mma3_f8_if(uint32_t issue, uint32_t d0, uint32_t d1, uint32_t d2, uint64_t a_desc,
                                           uint64_t b0, uint64_t b1, uint64_t b2, uint32_t idesc,
                                           uint32_t accumulate) {
    FX_MMA3("f8f6f4");
}
#undef FX_MMA3
// Two or three MMAs sharing one A tile through the A collector, each with its own accumulate flag
// (z-plane fold: the first MMA into a block starts it).
#define FX_MMAZ2(KIND)                                                                                          \
    asm volatile(                                                                                               \
        "{\n\t.reg .pred p0, p1, q;\n\tsetp.ne.b32 p0, %5, 0;\n\tsetp.ne.b32 p1, %6, 0;\n\t"                  \
        "setp.ne.b32 q, %7, 0;\n\t"                                                                              \
        "@q tcgen05.mma.cta_group::1.kind::" KIND ".collector::a::fill [%0], %2, %3, %8, p0;\n\t"              \
        "@q tcgen05.mma.cta_group::1.kind::" KIND ".collector::a::lastuse [%1], %2, %4, %8, p1;\n\t}"          \
        ::"r"(d0), "r"(d1), "l"(a_desc), "l"(b0), "l"(b1), "r"(acc0), "r"(acc1), "r"(issue), "r"(idesc)      \
        : "memory")
#define FX_MMAZ3(KIND)                                                                                          \
    asm volatile(                                                                                               \
        "{\n\t.reg .pred p0, p1, p2, q;\n\tsetp.ne.b32 p0, %7, 0;\n\tsetp.ne.b32 p1, %8, 0;\n\t"            \
        "setp.ne.b32 p2, %9, 0;\n\tsetp.ne.b32 q, %10, 0;\n\t"                                                 \
        "@q tcgen05.mma.cta_group::1.kind::" KIND ".collector::a::fill [%0], %3, %4, %11, p0;\n\t"             \
        "@q tcgen05.mma.cta_group::1.kind::" KIND ".collector::a::use [%1], %3, %5, %11, p1;\n\t"              \
        "@q tcgen05.mma.cta_group::1.kind::" KIND ".collector::a::lastuse [%2], %3, %6, %11, p2;\n\t}"         \
        ::"r"(d0), "r"(d1), "r"(d2), "l"(a_desc), "l"(b0), "l"(b1), "l"(b2), "r"(acc0), "r"(acc1), "r"(acc2), \
        "r"(issue), "r"(idesc)                                                                                  \
        : "memory")
__device__ __forceinline__ void mmaz2_f16_if(uint32_t issue, uint32_t d0, uint32_t d1, uint64_t a_desc, uint64_t b0,
                                             uint64_t b1, uint32_t idesc, uint32_t acc0, uint32_t acc1) {
    FX_MMAZ2("f16");
}
__device__ __forceinline__ void mmaz2_f8_if(uint32_t issue, uint32_t d0, uint32_t d1, uint64_t a_desc, uint64_t b0,
                                            uint64_t b1, uint32_t idesc, uint32_t acc0, uint32_t acc1) {
    FX_MMAZ2("f8f6f4");
}
__device__ __forceinline__ void mmaz3_f16_if(uint32_t issue, uint32_t d0, uint32_t d1, uint32_t d2, uint64_t a_desc,
                                             uint64_t b0, uint64_t b1, uint64_t b2, uint32_t idesc, uint32_t acc0,
                                             uint32_t acc1, uint32_t acc2) {
    FX_MMAZ3("f16");
}
__device__ __forceinline__ void mmaz3_f8_if(uint32_t issue, uint32_t d0, uint32_t d1, uint32_t d2, uint64_t a_desc,
                                            uint64_t b0, uint64_t b1, uint64_t b2, uint32_t idesc, uint32_t acc0,
                                            uint32_t acc1, uint32_t acc2) {
    FX_MMAZ3("f8f6f4");
}
#undef FX_MMAZ2
#undef FX_MMAZ3
__device__ __forceinline__ void mma_commit_if(uint32_t issue, uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %1, 0;\n\t"
        "@q tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar),
        "r"(issue)
        : "memory");
}

// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// 32 lanes x 32 columns of 32-bit: thread i of the warp gets lane (base_lane + i), columns c..c+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 columns of 32-bit.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Same 16-column load without the wait: several loads may be in flight before one tmem_wait().
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Ties 16 destination registers of earlier tcgen05.ld to a point after tmem_wait(), so the
// compiler cannot move any use of them above the wait.
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])::"memory");
}

// Shared-memory matrix descriptor, K-major, no swizzle ("interleaved" canonical layout):
// core matrices of 8 rows x 16 bytes, rows of one core matrix 16 B apart, the two K-halves of
// one MMA `lbo` bytes apart, consecutive 8-row groups `sbo` bytes apart. Layout type 0 and
// version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version for tcgen05
    return d;                             // base offset 0, lbo mode 0, layout type 0 (no swizzle)
}

// Instruction descriptor: f32 accumulate, K-major A and B, dense.
//   kind::f16      : a/b format 0 = f16, 1 = bf16
//   kind::f8f6f4   : a/b format 0 = e4m3
__host__ __device__ constexpr uint32_t instr_desc(int M, int N, int optype) {
    return (1u << 4)                                                  // D format f32
           | ((optype == kOpBF16 ? 1u : 0u) << 7)                     // A format
           | ((optype == kOpBF16 ? 1u : 0u) << 10)                    // B format
           | (static_cast<uint32_t>(N >> 3) << 17)                    // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);                   // M / 16
}

// ---- small numeric helpers ---------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
// Two floats -> two f16 (round to nearest, saturated to +-65504 so a large value never
// becomes inf).
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
    a = fminf(fmaxf(a, -65504.f), 65504.f);
    b = fminf(fmaxf(b, -65504.f), 65504.f);
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
// Eight floats -> one 16-byte cell of 16-bit values (bf16 or f16).
__device__ __forceinline__ uint4 pack_cell16(const float* v, int optype) {
    uint4 w;
    if (optype == kOpF16) {
        w.x = pack_f16x2(v[0], v[1]);
        w.y = pack_f16x2(v[2], v[3]);
        w.z = pack_f16x2(v[4], v[5]);
        w.w = pack_f16x2(v[6], v[7]);
    } else {
        w.x = pack_bf16x2(v[0], v[1]);
        w.y = pack_bf16x2(v[2], v[3]);
        w.z = pack_bf16x2(v[4], v[5]);
        w.w = pack_bf16x2(v[6], v[7]);
    }
    return w;
}
// Byte offset of padded voxel (zp, yp, xp)'s cell in a stride-2 conv's phase-split copy: one
// sub-volume per parity of the axes in mask m (bit 2 z, bit 1 y, bit 0 x), phase index = those
// parities in z, y, x order, each sub-volume padded pHp x pWp rows (the conv's output grid + 2)
// and ps bytes apart; a halved axis indexes by p >> 1, a full one by p.
__device__ __forceinline__ int64_t phase_cell_offset(int m, int zp, int yp, int xp, int pHp, int pWp, int64_t ps) {
    int phi = 0;
    if (m & 4) {
        phi = zp & 1;
        zp >>= 1;
    }
    if (m & 2) {
        phi = (phi << 1) | (yp & 1);
        yp >>= 1;
    }
    if (m & 1) {
        phi = (phi << 1) | (xp & 1);
        xp >>= 1;
    }
    return phi * ps + ((static_cast<int64_t>(zp) * pHp + yp) * pWp + xp) * 16;
}
// v rounded to the 16-bit operand type (round to nearest; f16 saturated as pack_f16x2 does).
__device__ __forceinline__ float round16(float v, int optype) {
    if (optype == kOpF16) return __half2float(__float2half_rn(fminf(fmaxf(v, -65504.f), 65504.f)));
    return __bfloat162float(__float2bfloat16_rn(v));
}
// The first conv's input cells for the three x taps v[0..2] (x - 1, x, x + 1) as two 16-bit terms,
// hi = round16(v) and lo = round16(v - hi) (v - hi is exact in f32), so hi + lo carries v to about
// twice the type's precision: cell 0 = [hi x3, lo x3, 0, 0] (multiplied by the 16-bit weights),
// cell 1 = [hi x3, 0 x5] (multiplied by the weights' rounding residues).
__device__ __forceinline__ void first_layer_cells(const float (&v)[3], int optype, uint4& c0, uint4& c1) {
    float hi[3], lo[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        hi[k] = round16(v[k], optype);
        lo[k] = v[k] - hi[k];
    }
    const float a[8] = {hi[0], hi[1], hi[2], lo[0], lo[1], lo[2], 0.f, 0.f};
    const float b[8] = {hi[0], hi[1], hi[2], 0.f, 0.f, 0.f, 0.f, 0.f};
    c0 = pack_cell16(a, optype);
    c1 = pack_cell16(b, optype);
}
// Eight floats -> one 16-byte cell of f16, round to nearest, saturated to +-65504 (one
// cvt.rn.satfinite.f16x2.f32 per pair; the first value of a pair lands in the low half).
__device__ __forceinline__ uint4 pack_cell_f16_sat(const float* v) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(w[i]) : "f"(v[2 * i + 1]), "f"(v[2 * i]));
    return make_uint4(w[0], w[1], w[2], w[3]);
}
// Four floats -> four e4m3 bytes (satfinite), little-endian in one u32.
__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
    __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
    __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// One 16-byte cell of eight 16-bit values (bf16 or f16) -> floats.
__device__ __forceinline__ void unpack_cell16(const uint4 w, int optype, float (&f)[8]) {
    if (optype == kOpF16) {
        const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 t = __half22float2(h[i]);
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    } else {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 t = __bfloat1622float2(h[i]);
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
}

}  // namespace fxk
