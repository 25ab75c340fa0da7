// Shared device helpers of the B200 VQ runtime (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "../../include/vqb.h"

namespace vqb {

constexpr int kWarp = 32;

// ---------------------------------------------------------------- numbers

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float2 h2x2f(uint32_t w) {
  __half2 v = *reinterpret_cast<__half2*>(&w);
  return __half22float2(v);
}

// Load one input element as the kernel's fp32 working value.  When
// narrow_f16 is set the value first takes the fp16 rounding the reference
// applies to x (host cast in vq_switch.py:5301-5308, in-kernel `(half)` in the
// dense kernels, vq_switch.py:2319-2327).
__device__ __forceinline__ float load_x(const void* x, int64_t i, int dtype, bool narrow_f16) {
  float v;
  if (dtype == VQB_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
  else if (dtype == VQB_F16) return __half2float(reinterpret_cast<const __half*>(x)[i]);
  else v = reinterpret_cast<const float*>(x)[i];
  if (narrow_f16) v = __half2float(__float2half_rn(v));
  return v;
}

// Store an fp32 accumulator.  round_f16_first reproduces the reference MoE
// output path: the kernel writes fp16, the module casts to x's dtype
// (vq_switch.py:5423), i.e. two roundings.
__device__ __forceinline__ void store_y(void* y, int64_t i, float acc, int dtype, bool round_f16_first) {
  if (round_f16_first) acc = __half2float(__float2half_rn(acc));
  if (dtype == VQB_BF16) reinterpret_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(acc);
  else if (dtype == VQB_F16) reinterpret_cast<__half*>(y)[i] = __float2half_rn(acc);
  else reinterpret_cast<float*>(y)[i] = acc;
}

// ------------------------------------------------- programmatic dependent launch

// Wait until the kernel before this one on the stream has finished and its
// writes are visible.  A kernel launched with launch_pdl (vqb_internal.h) calls
// this before its first global access; without the launch attribute it
// returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Let the next kernel on the stream start its CTAs (it still waits for this
// one's completion in its own pdl_wait).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------ global loads

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

// ---------------------------------------------------------------- bit walk

// Sequential reader of one row's packed code stream (vq_pack v1: code j at
// bits [j*BITS, (j+1)*BITS) of the little-endian word stream).  Words are
// fetched 16 bytes at a time when the row is 16-byte aligned (VEC) and held in
// a 64-bit window, so each word is read from memory once.
template <bool VEC>
struct BitWalker {
  const uint32_t* p;  // next word (scalar) or next 16-byte chunk (VEC)
  uint32_t q[4];
  int qi;             // next unread word of q
  uint64_t buf;
  int nb;             // valid bits in buf

  __device__ __forceinline__ uint32_t next_word() {
    if (VEC) {
      if (qi == 4) {
        uint4 v = ldg_stream_v4(p);
        p += 4;
        q[0] = v.x; q[1] = v.y; q[2] = v.z; q[3] = v.w;
        qi = 0;
      }
      uint32_t w = q[0];
      // rotate instead of dynamic indexing so q stays in registers
      q[0] = q[1]; q[1] = q[2]; q[2] = q[3];
      ++qi;
      return w;
    } else {
      return ldg_stream_u32(p++);
    }
  }

  // Position at bit `bit0` of the row starting at `row`.
  __device__ __forceinline__ void init(const uint32_t* row, int64_t bit0) {
    int64_t w = bit0 >> 5;
    int sh = static_cast<int>(bit0 & 31);
    if (VEC) {
      p = row + (w & ~int64_t(3));
      qi = 4;
      int skip = static_cast<int>(w & 3);
      for (int i = 0; i < skip; ++i) next_word();
    } else {
      p = row + w;
    }
    buf = next_word() >> sh;
    nb = 32 - sh;
  }

  __device__ __forceinline__ uint32_t next(int bits, uint32_t mask) {
    if (nb < bits) {
      buf |= static_cast<uint64_t>(next_word()) << nb;
      nb += 32;
    }
    uint32_t c = static_cast<uint32_t>(buf) & mask;
    buf >>= bits;
    nb -= bits;
    return c;
  }
};

// BitWalker with one 16-byte load in flight ahead of the one being consumed,
// so a long sequential walk never waits on a load it could have issued
// earlier.  Rows must be 16-byte aligned with a multiple of 4 words; loads
// past the row's end are not issued (they read as zero).
struct PrefetchWalker {
  const uint4* p;     // next chunk to request
  const uint4* end;   // one past the row's last chunk
  uint4 cur, nxt;
  int qi;             // next word of cur
  uint64_t buf;
  int nb;

  __device__ __forceinline__ uint4 fetch() {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (p < end) v = ldg_stream_v4(p);
    ++p;
    return v;
  }
  __device__ __forceinline__ uint32_t next_word() {
    if (qi == 4) {
      cur = nxt;
      nxt = fetch();
      qi = 0;
    }
    const uint32_t w = qi == 0 ? cur.x : (qi == 1 ? cur.y : (qi == 2 ? cur.z : cur.w));
    ++qi;
    return w;
  }
  // start at word 0 of a row of `row_words` words (a multiple of 4)
  __device__ __forceinline__ void init(const uint32_t* row, int row_words) {
    p = reinterpret_cast<const uint4*>(row);
    end = p + row_words / 4;
    cur = fetch();
    nxt = fetch();
    qi = 0;
    buf = next_word();
    nb = 32;
  }
  __device__ __forceinline__ uint32_t next(int bits, uint32_t mask) {
    if (nb < bits) {
      buf |= static_cast<uint64_t>(next_word()) << nb;
      nb += 32;
    }
    const uint32_t c = static_cast<uint32_t>(buf) & mask;
    buf >>= bits;
    nb -= bits;
    return c;
  }
};

}  // namespace vqb
