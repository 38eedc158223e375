// p8_format.h -- the Pingala-8 slot layout, shared by host and device code.
//
// Same bytes as the reference contract (ggml-vr-native.h CU:1-51, vr49.cuh CU:2519-2543); written from scratch.
//   [0, 2064)       header: A u32[256] @0 (int8x4 codebook), B u32[256] @1024 (= A), c u32 @2048 (coset int8x4),
//                   NS = 108 @2052, TRL = 2 @2056, word 515 @2060
//   M @2064         u32 per tile (g * nb + b): payload word offset | class << 29
//   S @2064 + 4 nt  fp16 [b][rows] (sorted rows)
//   D @align16(2064 + 68 nt)  per tile: [hs][i >> 1][lane j][i & 1] u32; lane j = tile row j, step k holds chunk
//                   t = (j + k) & 31 (4 columns 4t..4t+3 of the 128-column half-slice hs)
//   top-down from the end (CU:30-37): E delta (rows u16[nd] | cols u16[nd] | vals f32[nd]), C c16 fp16[K],
//   P prm int16[rows] (sorted -> original), Q pinv int16[rows], SG int8[256] Hadamard signs, trailer 32 B.
#pragma once
#include <stddef.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define P8_HD __host__ __device__ __forceinline__
#else
#define P8_HD inline
#endif

namespace p8 {

constexpr uint32_t kMagic0 = 0x4E525656u;  // "VVRN"
constexpr uint32_t kMagic1 = 0x31354952u;  // "RI51"
constexpr uint32_t kNS = 108u;             // Pingala-8: 8 gana states, u_t = z_t ^ u_{t-1} ^ u_{t-3}, h_t = u_{t-2}
constexpr uint32_t kTRL = 2u;
constexpr uint32_t kVR3Tag = 0x56523300u;  // VR3 file word 515 | class (llama-vr3.h)
constexpr size_t kHdrBytes = 2064;
constexpr int kMaxRows = 32767;            // int16 prm (loader CU:3481)

// per-class field widths (bits per 4-weight chunk and stage), shifts and words per lane per half-slice
P8_HD constexpr int W1(int c) { return c == 0 ? 0 : c == 1 ? 4 : c == 2 ? 6 : 8; }
P8_HD constexpr int W2(int c) { return c == 4 ? 2 : c == 5 ? 4 : c >= 6 ? 8 : 0; }
P8_HD constexpr int W3(int c) { return c == 7 ? 8 : 0; }
P8_HD constexpr int SH1(int c) { return c == 4 ? 2 : c == 5 ? 3 : c == 6 ? 2 : c == 7 ? 4 : 0; }
P8_HD constexpr int SH2(int c) { return c == 7 ? 2 : 0; }
P8_HD constexpr int NW(int c) { return W1(c) + W2(c) + W3(c); }
P8_HD constexpr int NST(int c) { return c == 0 ? 0 : c <= 3 ? 1 : c <= 6 ? 2 : 3; }
// coset multiplicity: h c is added to every stage, so the coset term carries sum_s 2^SH_s
P8_HD constexpr int MC(int c) { return (1 << SH1(c)) + (W2(c) ? (1 << SH2(c)) : 0) + (W3(c) ? 1 : 0); }

P8_HD constexpr size_t a16(size_t n) { return (n + 15) & ~(size_t)15; }
P8_HD constexpr size_t offS(size_t nt) { return kHdrBytes + 4 * nt; }
P8_HD constexpr size_t offD(size_t nt) { return (kHdrBytes + 68 * nt + 15) & ~(size_t)15; }

struct SideOffsets {
    size_t E, C, P, Q, SG, T;
};
P8_HD SideOffsets side_offsets(size_t n, size_t rows, size_t K, size_t nd) {
    SideOffsets o;
    o.T = n - 32;
    o.SG = o.T - 256;
    o.Q = (o.SG - 2 * rows) & ~(size_t)15;
    o.P = (o.Q - 2 * rows) & ~(size_t)15;
    o.C = (o.P - 2 * K) & ~(size_t)15;
    o.E = (o.C - 8 * nd) & ~(size_t)15;
    return o;
}
P8_HD size_t slot_need(size_t kbytes, size_t rows, size_t K, size_t nd) {
    return a16(kbytes) + a16(8 * nd) + a16(2 * K) + 2 * a16(2 * rows) + 256 + 32 + 64;
}

struct Trailer {
    uint32_t magic0, magic1, kbytes, nd, rows, K, ns, version;
};

// Pingala-8 trellis over 32 chunks in chunk order: input bit t = z_t (stage-1 MSB of chunk t); output bit t = h_t.
// u = z ^ (u << 1) ^ (u << 3) is solved by prefix doubling (u has no bits below 0: the state resets per half-slice).
P8_HD uint32_t pingala8_h(uint32_t z) {
    uint32_t u = z;
    u ^= (u << 1) ^ (u << 3);
    u ^= (u << 2) ^ (u << 6);
    u ^= (u << 4) ^ (u << 12);
    u ^= (u << 8) ^ (u << 24);
    u ^= u << 16;
    return u << 2;
}

P8_HD float half_bits_to_float(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t f;
    if (e == 0) {
        if (m == 0) {
            f = s;
        } else {  // subnormal: normalise
            int sh = 0;
            uint32_t mm = m;
            while (!(mm & 0x400u)) { mm <<= 1; ++sh; }
            f = s | ((uint32_t)(113 - sh) << 23) | ((mm & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        f = s | 0x7f800000u | (m << 13);
    } else {
        f = s | ((e + 112u) << 23) | (m << 13);
    }
    union { uint32_t u; float f; } cv;
    cv.u = f;
    return cv.f;
}

}  // namespace p8
