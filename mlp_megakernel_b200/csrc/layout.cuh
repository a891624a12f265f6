// Shared-memory operand layouts for tcgen05 UMMA (fp16 operands).
//
// Every operand tile is stored as "chunks": a chunk is ROWS rows of
// CHUNK elements of the contiguous dimension (CHUNK = min(64, extent)), with
// a row pitch of CHUNK*2 bytes and the matching TMA/UMMA swizzle (128B for a
// 128-byte pitch, 64B for 64, 32B for 32).  Chunks of one operand follow each
// other.  This is exactly what a TMA tiled load with box {CHUNK, ROWS} and the
// same swizzle writes, so the same layout serves TMA loads, TMA stores and the
// epilogue's st.shared of activations.
//
//  * K-major A (activations, [rows=M tile][K]): the contiguous dim is K.
//  * MN-major B (weights as stored by the caller, [K][N], N contiguous): the
//    contiguous dim is N; rows are K.
#pragma once
#include <cstdint>

namespace mlpk {

__host__ __device__ constexpr int chunk_elems(int extent) { return extent < 64 ? extent : 64; }
__host__ __device__ constexpr int pitch_bytes(int extent) { return chunk_elems(extent) * 2; }
// UMMA smem-descriptor layout code for a given row pitch (swizzle width).
__host__ __device__ constexpr uint32_t umma_layout_code(int pitch) {
  return pitch == 128 ? 2u : pitch == 64 ? 4u : 6u;  // SW128 / SW64 / SW32
}
// Bytes of an operand tile with `rows` rows and contiguous extent `extent`.
__host__ __device__ constexpr int tile_bytes(int rows, int extent) { return rows * extent * 2; }
__host__ __device__ constexpr int align_up(int v, int a) { return (v + a - 1) / a * a; }

// Byte offset of the 16-byte unit `unit` (8 fp16) of row `row` inside a chunk
// whose base is aligned to the swizzle repeat (1024 B covers every mode).
template <int PITCH>
__device__ __forceinline__ uint32_t swz_off(uint32_t row, uint32_t unit) {
  constexpr uint32_t mask = PITCH / 16 - 1;  // 7 / 3 / 1
  uint32_t o = row * PITCH + unit * 16;
  return o ^ (((o >> 7) & mask) << 4);
}

// 64-bit UMMA shared-memory descriptor (sm_100 format: version bit 46 = 1).
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes, uint32_t layout_code) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout_code & 7) << 61;
  return d;
}

// Instruction descriptor, kind::f16: A,B fp16, D fp32, A K-major, B MN-major.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                                    // D format: f32
         | (0u << 7) | (0u << 10)                     // A, B format: f16
         | (static_cast<uint32_t>(a_mn_major) << 15)  // A major
         | (static_cast<uint32_t>(b_mn_major) << 16)  // B major
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Instruction descriptor, kind::tf32: A, B tf32 (format 2), D fp32.
__host__ __device__ constexpr uint32_t make_idesc_tf32(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                                    // D format: f32
         | (2u << 7) | (2u << 10)                     // A, B format: tf32
         | (static_cast<uint32_t>(a_mn_major) << 15)  // A major
         | (static_cast<uint32_t>(b_mn_major) << 16)  // B major
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Byte offset of K-step `k` (16 elements of K) inside a K-major operand with
// `ROWS` rows and K extent `KEXT` (see the chunk layout above).
template <int ROWS, int KEXT>
__host__ __device__ constexpr uint32_t kmajor_koff(int k) {
  return (k * 16 / chunk_elems(KEXT)) * (ROWS * pitch_bytes(KEXT)) +
         (k * 16 % chunk_elems(KEXT)) * 2;
}
// Byte offset of K-step `k` inside an MN-major operand [K rows][NEXT cols].
template <int NEXT>
__host__ __device__ constexpr uint32_t mnmajor_koff(int k) {
  return k * 16 * pitch_bytes(NEXT);
}
// Base descriptors: the K-step descriptor is base + (koff >> 4) (the start
// address field is the low 14 bits; operands live below 256 KB, no carry).
template <int KEXT>
__device__ __forceinline__ uint64_t kmajor_base_desc(uint32_t base) {
  return make_sdesc(base, 16, 8 * pitch_bytes(KEXT), umma_layout_code(pitch_bytes(KEXT)));
}
template <int KROWS, int NEXT>
__device__ __forceinline__ uint64_t mnmajor_base_desc(uint32_t base) {
  return make_sdesc(base, KROWS * pitch_bytes(NEXT), 8 * pitch_bytes(NEXT),
                    umma_layout_code(pitch_bytes(NEXT)));
}

// MN-major tf32 operand [K rows][N cols] (fp32, N contiguous) stored as
// chunks of 32 columns x KROWS rows (128-byte rows).  For 32-bit MN-major
// operands the tensor core takes one swizzle only: 128 bytes with 32-byte
// atoms (layout code 1), where 32-byte granule g of row r sits at g ^ (r % 4)
// -- what a TMA load with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B writes.  A K
// group is 4 rows (SBO 512 B); chunks follow each other (LBO).
template <int KROWS>
__device__ __forceinline__ uint64_t mnmajor_tf32_base_desc(uint32_t base) {
  return make_sdesc(base, KROWS * 128, 4 * 128, 1u);
}

// Descriptor for K-step `k` (16 elements of K) of a K-major operand with
// `rows` rows and K extent `kext`, stored as chunks (see above).
template <int ROWS, int KEXT>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int k) {
  constexpr int C = chunk_elems(KEXT);
  constexpr int P = pitch_bytes(KEXT);
  const int kel = k * 16;
  const uint32_t addr = base + (kel / C) * (ROWS * P) + (kel % C) * 2;
  return make_sdesc(addr, 16, 8 * P, umma_layout_code(P));
}

// Descriptor for K-step `k` of an MN-major operand [K rows][NEXT cols]
// (N contiguous) stored as chunks of CHUNK columns x KROWS rows.
template <int KROWS, int NEXT>
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int k) {
  constexpr int P = pitch_bytes(NEXT);
  const uint32_t addr = base + k * 16 * P;
  return make_sdesc(addr, KROWS * P, 8 * P, umma_layout_code(P));
}

}  // namespace mlpk
