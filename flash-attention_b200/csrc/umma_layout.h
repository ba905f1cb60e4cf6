// Shared-memory tile layouts and tcgen05 (UMMA) descriptors.
//
// The reference stages tiles in 8 x 64-element atoms of 128-byte rows with an XOR
// swizzle of 16-byte chunks (src/tensor_core/swizzle.cuh:5-28, src/loadstore/copy_srm.cuh:14-30).
// Here the same idea is expressed in the layout that TMA writes and tcgen05.mma
// reads directly: rows of SW bytes (SW = 128, or 64 when a row holds only 32
// 16-bit elements), 8-row atoms of 8*SW bytes, 16-byte chunk index XOR row%8
// (SW=128) or XOR (row%8)/2 (SW=64).  A tile of R rows x D columns is split along
// D into D*2/SW column chunks, each a dense R x SW-byte region.
//
// Everything here is plain integer arithmetic usable on the host (unit tests
// check the bit fields) and on the device.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define FA_HD __host__ __device__ __forceinline__
#else
#define FA_HD inline
#endif

namespace fa {

enum : uint32_t {
  kLayoutSwizzleNone = 0,
  kLayoutSwizzle128B = 2,
  kLayoutSwizzle64B = 4,
  kLayoutSwizzle32B = 6,
};

// Bytes per swizzled row for a head dimension of `d` 16-bit elements.
FA_HD constexpr uint32_t swizzle_bytes(int d) { return d * 2 >= 128 ? 128u : static_cast<uint32_t>(d * 2); }

FA_HD constexpr uint32_t layout_type_for(uint32_t sw_bytes) {
  return sw_bytes == 128 ? kLayoutSwizzle128B : (sw_bytes == 64 ? kLayoutSwizzle64B : kLayoutSwizzle32B);
}

// Byte offset of element (row, col) of a 16-bit tile with `rows` rows stored as
// column chunks of SW-byte swizzled rows.  This is what TMA produces for a box of
// SW/2 columns x `rows` rows at chunk base row*SW, and what UMMA expects.
FA_HD constexpr uint32_t tile_offset_bytes(uint32_t row, uint32_t col, uint32_t rows, uint32_t sw) {
  const uint32_t chunk = (col * 2) / sw;
  const uint32_t byte_in_row = (col * 2) % sw;
  const uint32_t c16 = byte_in_row / 16;
  const uint32_t xor_mask = sw == 128 ? (row % 8) : (sw == 64 ? ((row % 8) / 2) : ((row % 8) / 4));
  const uint32_t c16_sw = c16 ^ xor_mask;
  return chunk * rows * sw + row * sw + c16_sw * 16 + (byte_in_row % 16);
}

// tcgen05 shared-memory matrix descriptor (64 bits):
//   [0,14)  start address >> 4      [16,30) leading byte offset >> 4
//   [32,46) stride byte offset >> 4 [46,48) version = 1 (sm_100)
//   [49,52) base offset = 0 (atoms are 1024-byte aligned)   [52] LBO mode = 0
//   [61,64) layout type (swizzle mode)
FA_HD constexpr uint64_t make_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                        uint32_t layout_type) {
  return (static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu)) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(layout_type & 0x7u) << 61);
}

// K-major operand (rows = M or N, contiguous = K), swizzled rows of SW bytes:
// 8-row groups are SBO = 8*SW apart; LBO is unused by swizzled K-major layouts
// and set to 16 bytes.  One MMA consumes K=16 elements = 32 bytes of a row, so
// step kk of the K loop starts at chunk (kk*32)/SW, byte (kk*32)%SW of the row.
FA_HD constexpr uint64_t kmajor_desc(uint32_t tile_base, uint32_t rows, uint32_t sw, uint32_t kk) {
  const uint32_t kbyte = kk * 32u;
  const uint32_t addr = tile_base + (kbyte / sw) * rows * sw + (kbyte % sw);
  return make_smem_desc(addr, 16u, 8u * sw, layout_type_for(sw));
}

// MN-major operand (rows = K, contiguous = N), the V tile of O += P V:
// within a chunk, 8 K-rows are SBO = 8*SW apart; consecutive N-chunks of SW/2
// elements are LBO = rows*SW apart.  Step kk of the K loop moves 16 rows.
FA_HD constexpr uint64_t mnmajor_desc(uint32_t tile_base, uint32_t rows, uint32_t sw, uint32_t kk) {
  const uint32_t addr = tile_base + kk * 16u * sw;
  return make_smem_desc(addr, rows * sw, 8u * sw, layout_type_for(sw));
}

// tcgen05 instruction descriptor for kind::f16 (32 bits):
//   [4,6) D format (1 = f32)  [7,10) A format  [10,13) B format (0 = f16, 1 = bf16)
//   [15] A major  [16] B major (0 = K, 1 = MN)  [17,23) N >> 3  [24,29) M >> 4
FA_HD constexpr uint32_t make_idesc_f16(bool bf16, int m, int n, bool a_mn_major, bool b_mn_major) {
  const uint32_t fmt = bf16 ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | ((static_cast<uint32_t>(n) >> 3) << 17) |
         ((static_cast<uint32_t>(m) >> 4) << 24);
}

}  // namespace fa
