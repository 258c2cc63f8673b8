// wire.cuh — the pipeline wire format (INTEGER_LLM/pipeline/src/codec.rs) with
// its CRC-32 computed on the GPU for frames whose payload lives in HBM.
//
// Frame (codec.rs:1-13, :86-111), all integers little-endian:
//   "IINTPIPE" | version, theta_v_hash, request_id, sequence_id, stage_id,
//   token_position, payload_len, flags, reserved (9 x u64) | crc32 (u32)
//   | payload (int16 values, 2 bytes each) | zero padding to a multiple of 8.
// The CRC is the one of the crc32fast crate the reference uses (version 1.3,
// Cargo.toml of the pipeline crate): CRC-32/ISO-HDLC, reflected polynomial
// 0xEDB88320, initial value and final XOR 0xFFFFFFFF (check value of
// "123456789" = 0xCBF43926), over the payload bytes only.
//
// Device CRC. The CRC register is affine in the data: with S(s, M) the
// register after feeding M from state s,
//   S(0, A || B) = S(0, B) xor S(0, A) * x^(8|B|)   (mod P, reflected bits)
// and crc(M) = S(0, M) xor 0xFFFFFFFF * x^(8|M|) xor 0xFFFFFFFF. Leading
// zero bytes leave S(0, .) at 0, so the data is treated as left-padded with
// zeros to whole blocks. Every thread runs the byte-table CRC over one chunk,
// shifts it by the bytes that follow it inside its block (one multiplication
// by a per-position power), the block XOR-reduces, and one thread shifts the
// block's value by the bytes of the blocks after it (powers x^(8B*2^k)) and
// XORs it into the result word.
#pragma once

#include <cstring>

#include "common.cuh"

namespace myl {

constexpr uint32_t CRC_POLY = 0xEDB88320u;  // reflected x^32 + x^26 + ... + 1
constexpr int CRC_THREADS = 256;
constexpr int CRC_CHUNK = 256;                       // bytes per thread
constexpr int64_t CRC_BLOCK = int64_t(CRC_THREADS) * CRC_CHUNK;
constexpr int CRC_POW_LEVELS = 48;                   // x^(8B * 2^k), k < 48

// a * b mod P in the reflected representation (bit 31 = x^0, bit 0 = x^31).
__host__ __device__ inline uint32_t gf2_mulmod(uint32_t a, uint32_t b) {
  uint32_t p = 0;
  for (int i = 0; i < 32; ++i) {
    if (a & (0x80000000u >> i)) p ^= b;
    b = (b & 1u) ? (b >> 1) ^ CRC_POLY : b >> 1;  // b * x
  }
  return p;
}

// x^(8 n) mod P (n bytes of zeros).
__host__ __device__ inline uint32_t gf2_x8n(uint64_t n) {
  uint32_t r = 0x80000000u;     // 1
  uint32_t base = 0x00800000u;  // x^8
  while (n) {
    if (n & 1) r = gf2_mulmod(r, base);
    base = gf2_mulmod(base, base);
    n >>= 1;
  }
  return r;
}

struct CrcTables {
  uint32_t pos[CRC_THREADS];        // x^(8 C (THREADS - 1 - t)): shift of chunk t in its block
  uint32_t pow[CRC_POW_LEVELS];     // x^(8 B 2^k)
};

inline void crc_tables_host(CrcTables* t) {
  for (int i = 0; i < CRC_THREADS; ++i) t->pos[i] = gf2_x8n(uint64_t(CRC_THREADS - 1 - i) * CRC_CHUNK);
  uint32_t p = gf2_x8n(uint64_t(CRC_BLOCK));
  for (int k = 0; k < CRC_POW_LEVELS; ++k) {
    t->pow[k] = p;
    p = gf2_mulmod(p, p);
  }
}

// Byte-table CRC update of state s (no initial value or final XOR).
inline uint32_t crc_raw_host(uint32_t s, const uint8_t* p, uint64_t n) {
  static uint32_t table[256];
  static bool init = false;
  if (!init) {
    for (uint32_t b = 0; b < 256; ++b) {
      uint32_t c = b;
      for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ CRC_POLY : c >> 1;
      table[b] = c;
    }
    init = true;
  }
  for (uint64_t i = 0; i < n; ++i) s = table[(s ^ p[i]) & 0xFFu] ^ (s >> 8);
  return s;
}

inline uint32_t crc32_host(const uint8_t* p, uint64_t n) {
  return crc_raw_host(0xFFFFFFFFu, p, n) ^ 0xFFFFFFFFu;
}

// out[0] ^= S(0, data) for data left-padded with `pad` zero bytes to
// nblocks * CRC_BLOCK bytes. out must start at 0.
__global__ void __launch_bounds__(CRC_THREADS)
    crc32_blocks_kernel(const uint8_t* __restrict__ data, uint64_t len, uint64_t pad,
                        uint64_t nblocks, CrcTables tabs, uint32_t* __restrict__ out) {
  __shared__ uint32_t table[256];
  __shared__ uint32_t part[CRC_THREADS / 32];
  {
    uint32_t c = threadIdx.x;
    for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ CRC_POLY : c >> 1;
    table[threadIdx.x] = c;
  }
  __syncthreads();
  for (uint64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    // chunk bytes [c0, c0 + CHUNK) of the padded stream = data[c0 - pad, ...)
    const int64_t c0 = int64_t(b) * CRC_BLOCK + int64_t(threadIdx.x) * CRC_CHUNK - int64_t(pad);
    const int64_t lo = c0 < 0 ? 0 : c0;
    const int64_t hi = c0 + CRC_CHUNK;  // <= len: the padding makes the stream end at len
    uint32_t s = 0;
    if (hi > lo) {
      if (lo == c0 && ((reinterpret_cast<uintptr_t>(data + lo) & 15) == 0)) {
        const uint4* q = reinterpret_cast<const uint4*>(data + lo);
#pragma unroll 1
        for (int v = 0; v < CRC_CHUNK / 16; ++v) {
          const uint4 w = __ldg(q + v);
          const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              s = table[(s ^ (words[e] >> (8 * k))) & 0xFFu] ^ (s >> 8);
        }
      } else {
        for (int64_t i = lo; i < hi; ++i) s = table[(s ^ data[i]) & 0xFFu] ^ (s >> 8);
      }
    }
    s = gf2_mulmod(s, tabs.pos[threadIdx.x]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s ^= __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t v = 0;
      for (int w = 0; w < CRC_THREADS / 32; ++w) v ^= part[w];
      uint64_t after = nblocks - 1 - b;  // blocks that follow this one
      for (int k = 0; after && k < CRC_POW_LEVELS; ++k, after >>= 1)
        if (after & 1) v = gf2_mulmod(v, tabs.pow[k]);
      atomicXor(out, v);
    }
    __syncthreads();
  }
}

// ---- host codec --------------------------------------------------------------
constexpr uint64_t WIRE_HEADER = 8 + 9 * 8 + 4;  // codec.rs:13

inline void wire_put_u64(uint8_t* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = uint8_t(v >> (8 * i));
}
inline uint64_t wire_get_u64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 0; i < 8; ++i) v |= uint64_t(p[i]) << (8 * i);
  return v;
}

inline uint64_t wire_frame_bytes(uint64_t n_values) {
  const uint64_t raw = WIRE_HEADER + 2 * n_values;
  return raw + ((8 - raw % 8) % 8);
}

}  // namespace myl
