// Block-scale quantizer kernels (HBM-bound): the MX formats (E4M3 / E5M2 / E2M1 codes + per-32 E8M0
// scales, rceil or floor rule) and NVFP4 (E2M1 + per-16 E4M3 + optional fp32 tensor scale), scale bytes
// written straight into the blocked (rm, rk, 32, 4, 4) layout.
//
// Work decomposition: one CTA owns a tile of 128 rows x 128 columns = one (MXFP8) or two
// (NVFP4) scale-factor atoms.  Every lane loads 16 consecutive elements (32 B of bf16 / 64 B of
// fp32; 8 lanes read one contiguous 256 B / 512 B row segment), reduces the block maximum
// (in-thread for NVFP4, one shuffle for MXFP8), converts, and stores 16 B (MXFP8) or 8 B
// (NVFP4) of codes.  Scale bytes are collected in shared memory in atom order and written once
// per CTA as whole 512-byte atoms, so every scale sector is written exactly once.  Short CTAs
// (32 KB of input) keep the tail of the last wave small.
#include "gemm_host.h"

#include <cuda_bf16.h>

#include <mutex>

namespace qk {

constexpr int Q_TILE_ROWS = 128;
constexpr int Q_TILE_COLS = 128;
constexpr int Q_THREADS = 256;
constexpr int Q_ITERS = 4;  // 32 rows per pass: 8 lanes x 16 elements cover one 128-column row segment

__device__ __forceinline__ uint32_t cvt4_e4m3(float a, float b, float c, float d) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}
__device__ __forceinline__ uint32_t cvt4_e5m2(float a, float b, float c, float d) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}
__device__ __forceinline__ uint32_t cvt8_e2m1(const float* v) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return r;
}
__device__ __forceinline__ float e4m3_to_float(uint32_t b) {
  uint32_t h;
  asm("{\n\t.reg .b16 s;\n\tcvt.u16.u32 s, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, s;\n\t}" : "=r"(h) : "r"(b & 0xFFu));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFFu)));
}

// 16 consecutive elements of a row: raw 16-byte words first (so that several rows' loads are
// in flight together), converted to fp32 afterwards
template <typename T> struct Raw16;
template <> struct Raw16<__nv_bfloat16> {
  uint4 w[2];
  __device__ __forceinline__ void load(const __nv_bfloat16* p) {
    w[0] = __ldg(reinterpret_cast<const uint4*>(p));
    w[1] = __ldg(reinterpret_cast<const uint4*>(p) + 1);
  }
  __device__ __forceinline__ void zero() { w[0] = w[1] = make_uint4(0, 0, 0, 0); }
  __device__ __forceinline__ void to_float(float (&v)[16]) const {
    const uint32_t u[8] = {w[0].x, w[0].y, w[0].z, w[0].w, w[1].x, w[1].y, w[1].z, w[1].w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[2 * i] = __uint_as_float(u[i] << 16);
      v[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
    }
  }
};
template <> struct Raw16<float> {
  float4 w[4];
  __device__ __forceinline__ void load(const float* p) {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = __ldg(reinterpret_cast<const float4*>(p) + i);
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __device__ __forceinline__ void to_float(float (&v)[16]) const {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[4 * i] = w[i].x; v[4 * i + 1] = w[i].y; v[4 * i + 2] = w[i].z; v[4 * i + 3] = w[i].w;
    }
  }
};

// max over |v| as an integer maximum of the sign-cleared bit patterns: orders like the floats
// and ranks NaN above infinity, so a NaN in the block survives the reduction (torch.amax
// propagates NaN).
__device__ __forceinline__ uint32_t absmax_bits16(const float (&v)[16]) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) m = max(m, __float_as_uint(v[i]) & 0x7FFFFFFFu);
  return m;
}

// One CTA quantises a 128-row x 128-column tile: exactly one (MXFP8) or two (NVFP4) scale
// atoms.  8 lanes cover a row segment (256 bytes of bf16), a warp covers 4 rows, the CTA 32
// rows per pass; the 4 passes are unrolled with all loads issued first.
// FLOOR selects the E8M0 rule of the MX formats: false = rceil, the exponent of amax / format_max rounded up
// (quack/blockscaled/quantize.py:267-282); true = floor, exponent(amax) - exponent(format_max) (:254-264, the only
// rule of MXFP4, :285-316).
template <typename T, int FORMAT, bool FLOOR>
__global__ void __launch_bounds__(Q_THREADS, 4)
quantize_blockscaled_kernel(const T* __restrict__ x, long long ldx, long long rows, long long k,
                            unsigned char* __restrict__ codes, long long ld_codes,
                            unsigned char* __restrict__ sf_blocked, long long rk_total,
                            const float* __restrict__ pts_ptr) {
  constexpr int VEC = FORMAT == QK_FMT_NVFP4 ? 16 : 32;
  constexpr int ATOMS = Q_TILE_COLS / (4 * VEC);  // scale atoms per tile: 1 (MX) / 2 (NV)
  __shared__ __align__(16) unsigned char sf_smem[ATOMS * 512];

  const int seg = threadIdx.x & 7;       // 16-element segment inside the 128-column tile row
  const int rsub = threadIdx.x >> 3;     // row inside a 32-row pass
  const long long row_base = static_cast<long long>(blockIdx.y) * Q_TILE_ROWS;
  const long long col = static_cast<long long>(blockIdx.x) * Q_TILE_COLS + seg * 16;
  const bool col_ok = col < k;

  for (int i = threadIdx.x; i < ATOMS * 512 / 16; i += Q_THREADS)
    reinterpret_cast<uint4*>(sf_smem)[i] = make_uint4(0, 0, 0, 0);

  float inv_pts = 1.f, pts = 1.f;
  if (FORMAT == QK_FMT_NVFP4 && pts_ptr != nullptr) {
    pts = __ldg(pts_ptr);
    inv_pts = __fdiv_rn(1.0f, pts);
  }

  Raw16<T> raw[Q_ITERS];
#pragma unroll
  for (int it = 0; it < Q_ITERS; ++it) {
    const long long row = row_base + it * 32 + rsub;
    // lanes outside the matrix still take part in the shuffles below (K % VEC == 0 keeps
    // the lanes of one block together) and skip their stores
    if (col_ok && row < rows) raw[it].load(x + row * ldx + col);
    else raw[it].zero();
  }
  __syncthreads();  // sf_smem is zeroed

#pragma unroll
  for (int it = 0; it < Q_ITERS; ++it) {
    const int r = it * 32 + rsub;
    const long long row = row_base + r;
    const bool ok = col_ok && row < rows;
    float v[16];
    raw[it].to_float(v);
    uint32_t mbits = absmax_bits16(v);
    if constexpr (FORMAT != QK_FMT_NVFP4) {
      mbits = max(mbits, __shfl_xor_sync(0xffffffffu, mbits, 1));
      const float amax = __uint_as_float(mbits);
      constexpr float FMT_MAX = FORMAT == QK_FMT_MXFP8_E4M3 ? 448.0f : FORMAT == QK_FMT_MXFP8_E5M2 ? 57344.0f : 6.0f;
      constexpr int FMT_MAX_POW2 = FORMAT == QK_FMT_MXFP8_E4M3 ? 8 : FORMAT == QK_FMT_MXFP8_E5M2 ? 15 : 2;
      uint32_t e;
      if constexpr (FLOOR) {
        // biased exponent field of amax, minus the exponent of the format's largest value
        const int p2 = static_cast<int>((mbits >> 23) & 0xFFu) - 127 - FMT_MAX_POW2;
        e = static_cast<uint32_t>(min(max(p2, -127), 128) + 127);
      } else {
        // biased E8M0 exponent of amax / format max, rounded up when the mantissa is non-zero
        const uint32_t rb = __float_as_uint(__fdiv_rn(amax, FMT_MAX));
        e = (rb >> 23) & 0xFFu;
        if (rb & 0x7FFFFFu) e += 1;
        e = min(e, 255u);
      }
      if (mbits > 0x7F800000u) e = 255u;  // NaN block
      // x / 2^(e-127) as an exact multiplication by the reciprocal power of two; e == 0
      // divides by 2^-126; e == 255 (scale = inf) multiplies by zero
      float rcp;
      if (e == 255u) rcp = 0.f;
      else if (e == 0u) rcp = __uint_as_float(253u << 23);
      else if (e == 254u) rcp = __uint_as_float(0x00400000u);  // 2^-127
      else rcp = __uint_as_float((254u - e) << 23);
      if constexpr (FORMAT == QK_FMT_MXFP4) {
        float y[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = v[i] * rcp;
        uint2 out;
        out.x = cvt8_e2m1(y);
        out.y = cvt8_e2m1(y + 8);
        if (ok) *reinterpret_cast<uint2*>(codes + row * ld_codes + (col >> 1)) = out;
      } else {
        uint4 out;
        if constexpr (FORMAT == QK_FMT_MXFP8_E4M3) {
          out.x = cvt4_e4m3(v[0] * rcp, v[1] * rcp, v[2] * rcp, v[3] * rcp);
          out.y = cvt4_e4m3(v[4] * rcp, v[5] * rcp, v[6] * rcp, v[7] * rcp);
          out.z = cvt4_e4m3(v[8] * rcp, v[9] * rcp, v[10] * rcp, v[11] * rcp);
          out.w = cvt4_e4m3(v[12] * rcp, v[13] * rcp, v[14] * rcp, v[15] * rcp);
        } else {
          out.x = cvt4_e5m2(v[0] * rcp, v[1] * rcp, v[2] * rcp, v[3] * rcp);
          out.y = cvt4_e5m2(v[4] * rcp, v[5] * rcp, v[6] * rcp, v[7] * rcp);
          out.z = cvt4_e5m2(v[8] * rcp, v[9] * rcp, v[10] * rcp, v[11] * rcp);
          out.w = cvt4_e5m2(v[12] * rcp, v[13] * rcp, v[14] * rcp, v[15] * rcp);
        }
        if (ok) *reinterpret_cast<uint4*>(codes + row * ld_codes + col) = out;
      }
      if (ok && (seg & 1) == 0) {
        const int kb = seg >> 1;  // scale column inside the tile: 0..3
        sf_smem[(r & 31) * 16 + (r >> 5) * 4 + kb] = static_cast<unsigned char>(e);
      }
    } else {
      const float amax = __uint_as_float(mbits);
      const float bs = __fdiv_rn(amax, 6.0f);
      const float t = pts_ptr != nullptr ? __fdiv_rn(bs, pts) : bs;
      const float tc = fminf(fmaxf(t, 0.015625f), 448.0f);
      uint16_t sfh;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(sfh) : "f"(0.f), "f"(tc));
      const uint32_t sfb = sfh & 0xFFu;
      const float recip = __fdiv_rn(inv_pts, e4m3_to_float(sfb));
      float y[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) y[i] = fminf(fmaxf(__fmul_rn(v[i], recip), -6.0f), 6.0f);
      uint2 out;
      out.x = cvt8_e2m1(y);
      out.y = cvt8_e2m1(y + 8);
      uint32_t sf_byte = sfb;
      if (mbits > 0x7F800000u) {
        // NaN block.  torch.clamp keeps the NaN (fminf / fmaxf above drop it): the scale byte is the E4M3
        // NaN, the reciprocal and every scaled element are NaN, and the reference's integer E2M1 encoder
        // (quack/blockscaled/quantize.py:165-207) maps that NaN pattern to code 4 whatever the element was.
        sf_byte = 0x7Fu;
        out.x = out.y = 0x44444444u;
      }
      if (ok) *reinterpret_cast<uint2*>(codes + row * ld_codes + (col >> 1)) = out;
      const int kb = seg;  // scale column inside the tile: 0..7
      if (ok) sf_smem[(kb >> 2) * 512 + (r & 31) * 16 + (r >> 5) * 4 + (kb & 3)] = static_cast<unsigned char>(sf_byte);
    }
  }
  __syncthreads();
  // write the tile's atoms (pad rows / columns stay zero); atoms past ceil(sf_k/4) are skipped
  const long long atom0 = static_cast<long long>(blockIdx.x) * ATOMS;
  unsigned char* dst = sf_blocked + (static_cast<long long>(blockIdx.y) * rk_total + atom0) * 512;
  if (threadIdx.x < ATOMS * 32) {
    const int atom = threadIdx.x >> 5;
    if (atom0 + atom < rk_total)
      reinterpret_cast<uint4*>(dst)[threadIdx.x] = reinterpret_cast<const uint4*>(sf_smem)[threadIdx.x];
  }
}

// ---- quantisation along dim 0 with a transposed result --------------------------------------------------
// x is (R, C) row-major; scale blocks run along R (down the columns).  The result is what the row quantizer
// gives for the transposed matrix: codes_t (C, R) row-major and blocked scales of a (C, R) operand, i.e.
// BlockScaledOperand.quantize(x, dim=-2) of the reference (quack/blockscaled/operand.py:718-783: "quantise
// the transposed copy and view back") without materialising the transposed high-precision copy.
// One CTA: a 128 (R) x 128 (C) tile.  The tile is read with coalesced 16-byte loads along C into shared
// memory; then a lane owns one column c and 32 consecutive rows (one MX block / two NVFP4 blocks): the lanes of
// a warp read consecutive c of the same row (conflict-free) and each writes 32 (fp8) or 16 (fp4) contiguous
// bytes of its output row.
__device__ __forceinline__ float tile_elem(const __nv_bfloat16* t, int i) { return __bfloat162float(t[i]); }
__device__ __forceinline__ float tile_elem(const float* t, int i) { return t[i]; }

template <int FORMAT, bool FLOOR>
__device__ __forceinline__ uint32_t mx_scale_exponent(uint32_t mbits) {
  constexpr float FMT_MAX = FORMAT == QK_FMT_MXFP8_E4M3 ? 448.0f : FORMAT == QK_FMT_MXFP8_E5M2 ? 57344.0f : 6.0f;
  constexpr int FMT_MAX_POW2 = FORMAT == QK_FMT_MXFP8_E4M3 ? 8 : FORMAT == QK_FMT_MXFP8_E5M2 ? 15 : 2;
  uint32_t e;
  if constexpr (FLOOR) {
    const int p2 = static_cast<int>((mbits >> 23) & 0xFFu) - 127 - FMT_MAX_POW2;
    e = static_cast<uint32_t>(min(max(p2, -127), 128) + 127);
  } else {
    const uint32_t rb = __float_as_uint(__fdiv_rn(__uint_as_float(mbits), FMT_MAX));
    e = (rb >> 23) & 0xFFu;
    if (rb & 0x7FFFFFu) e += 1;
    e = min(e, 255u);
  }
  if (mbits > 0x7F800000u) e = 255u;  // NaN block
  return e;
}
__device__ __forceinline__ float e8m0_reciprocal(uint32_t e) {
  if (e == 255u) return 0.f;                               // scale = inf
  if (e == 0u) return __uint_as_float(253u << 23);         // scale clamps to 2^-126
  if (e == 254u) return __uint_as_float(0x00400000u);      // 2^-127
  return __uint_as_float((254u - e) << 23);
}

constexpr int QT_TILE = 128;
template <typename T> struct QtPitch { static constexpr int value = QT_TILE + 16 / static_cast<int>(sizeof(T)); };

template <typename T, int FORMAT, bool FLOOR>
__global__ void __launch_bounds__(Q_THREADS)
quantize_blockscaled_t_kernel(const T* __restrict__ x, long long ldx, long long R, long long Ccols,
                              unsigned char* __restrict__ codes_t, long long ld_codes,
                              unsigned char* __restrict__ sf_blocked, long long rk_total,
                              const float* __restrict__ pts_ptr) {
  constexpr int VEC = FORMAT == QK_FMT_NVFP4 ? 16 : 32;
  constexpr int ATOMS = QT_TILE / (4 * VEC);
  constexpr bool FP4 = FORMAT == QK_FMT_NVFP4 || FORMAT == QK_FMT_MXFP4;
  constexpr int PITCH = QtPitch<T>::value;
  constexpr int EPC = 16 / static_cast<int>(sizeof(T));   // elements per 16-byte chunk
  extern __shared__ __align__(16) unsigned char qt_smem[];
  T* tile = reinterpret_cast<T*>(qt_smem);
  unsigned char* sf_smem = qt_smem + static_cast<size_t>(QT_TILE) * PITCH * sizeof(T);

  const long long r_base = static_cast<long long>(blockIdx.y) * QT_TILE;
  const long long c_base = static_cast<long long>(blockIdx.x) * QT_TILE;
  for (int i = threadIdx.x; i < ATOMS * 512 / 16; i += Q_THREADS)
    reinterpret_cast<uint4*>(sf_smem)[i] = make_uint4(0, 0, 0, 0);
  // load: rows outside the matrix and columns past C read as zeros
  constexpr int CHUNKS_PER_ROW = QT_TILE / EPC;
  for (int i = threadIdx.x; i < QT_TILE * CHUNKS_PER_ROW; i += Q_THREADS) {
    const int r = i / CHUNKS_PER_ROW, ch = i - r * CHUNKS_PER_ROW;
    const long long row = r_base + r, col = c_base + ch * EPC;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < R) {
      if (col + EPC <= Ccols) {
        v = __ldg(reinterpret_cast<const uint4*>(x + row * ldx + col));
      } else if (col < Ccols) {
        T tmp[EPC];
#pragma unroll
        for (int j = 0; j < EPC; ++j) tmp[j] = (col + j < Ccols) ? x[row * ldx + col + j] : T(0);
        v = *reinterpret_cast<const uint4*>(tmp);
      }
    }
    *reinterpret_cast<uint4*>(tile + r * PITCH + ch * EPC) = v;
  }
  float inv_pts = 1.f, pts = 1.f;
  if (FORMAT == QK_FMT_NVFP4 && pts_ptr != nullptr) {
    pts = __ldg(pts_ptr);
    inv_pts = __fdiv_rn(1.0f, pts);
  }
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
    const int c = (warp & 3) * 32 + lane;          // column of the tile = output row
    const int blk = (warp >> 2) + 2 * pass;        // 32-row block of the tile: 0..3
    const long long orow = c_base + c;
    const long long ocol = r_base + blk * 32;      // first logical element of this thread's 32 in the output row
    const bool ok = orow < Ccols && ocol < R;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = tile_elem(tile, (blk * 32 + j) * PITCH + c);
    uint32_t mb[2] = {0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      mb[0] = max(mb[0], __float_as_uint(v[j]) & 0x7FFFFFFFu);
      mb[1] = max(mb[1], __float_as_uint(v[16 + j]) & 0x7FFFFFFFu);
    }
    unsigned char* orow_ptr = codes_t + orow * ld_codes;
    if constexpr (FORMAT != QK_FMT_NVFP4) {
      const uint32_t e = mx_scale_exponent<FORMAT, FLOOR>(max(mb[0], mb[1]));
      const float rcp = e8m0_reciprocal(e);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= rcp;
      if (ok) {
        if constexpr (FP4) {
          *reinterpret_cast<uint4*>(orow_ptr + (ocol >> 1)) = make_uint4(cvt8_e2m1(v), cvt8_e2m1(v + 8), cvt8_e2m1(v + 16), cvt8_e2m1(v + 24));
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float* w = v + 16 * h;
            uint4 out;
            if constexpr (FORMAT == QK_FMT_MXFP8_E4M3) {
              out = make_uint4(cvt4_e4m3(w[0], w[1], w[2], w[3]), cvt4_e4m3(w[4], w[5], w[6], w[7]),
                               cvt4_e4m3(w[8], w[9], w[10], w[11]), cvt4_e4m3(w[12], w[13], w[14], w[15]));
            } else {
              out = make_uint4(cvt4_e5m2(w[0], w[1], w[2], w[3]), cvt4_e5m2(w[4], w[5], w[6], w[7]),
                               cvt4_e5m2(w[8], w[9], w[10], w[11]), cvt4_e5m2(w[12], w[13], w[14], w[15]));
            }
            *reinterpret_cast<uint4*>(orow_ptr + ocol + 16 * h) = out;
          }
        }
        sf_smem[(c & 31) * 16 + (c >> 5) * 4 + blk] = static_cast<unsigned char>(e);
      }
    } else {
      uint32_t words[4];
      uint32_t sfb2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float amax = __uint_as_float(mb[h]);
        const float bs = __fdiv_rn(amax, 6.0f);
        const float t = pts_ptr != nullptr ? __fdiv_rn(bs, pts) : bs;
        const float tc = fminf(fmaxf(t, 0.015625f), 448.0f);
        uint16_t sfh;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(sfh) : "f"(0.f), "f"(tc));
        uint32_t sfb = sfh & 0xFFu;
        const float recip = __fdiv_rn(inv_pts, e4m3_to_float(sfb));
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = fminf(fmaxf(__fmul_rn(v[16 * h + j], recip), -6.0f), 6.0f);
        words[2 * h] = cvt8_e2m1(y);
        words[2 * h + 1] = cvt8_e2m1(y + 8);
        if (mb[h] > 0x7F800000u) {   // NaN block: see the row quantizer
          sfb = 0x7Fu;
          words[2 * h] = words[2 * h + 1] = 0x44444444u;
        }
        sfb2[h] = sfb;
      }
      if (ok) {
        *reinterpret_cast<uint4*>(orow_ptr + (ocol >> 1)) = make_uint4(words[0], words[1], words[2], words[3]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int kb = blk * 2 + h;   // scale column inside the tile: 0..7
          sf_smem[(kb >> 2) * 512 + (c & 31) * 16 + (c >> 5) * 4 + (kb & 3)] = static_cast<unsigned char>(sfb2[h]);
        }
      }
    }
  }
  __syncthreads();
  const long long atom0 = static_cast<long long>(blockIdx.y) * ATOMS;
  unsigned char* dst = sf_blocked + (static_cast<long long>(blockIdx.x) * rk_total + atom0) * 512;
  if (threadIdx.x < ATOMS * 32) {
    const int atom = threadIdx.x >> 5;
    if (atom0 + atom < rk_total)
      reinterpret_cast<uint4*>(dst)[threadIdx.x] = reinterpret_cast<const uint4*>(sf_smem)[threadIdx.x];
  }
}

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&v)[16]) {
  Raw16<T> r;
  r.load(p);
  r.to_float(v);
}

template <typename T>
__global__ void __launch_bounds__(256) amax_kernel(const T* __restrict__ x, long long ldx, long long rows,
                                                   long long k, float* __restrict__ out) {
  // k % 16 == 0; every thread strides over 16-element groups
  const long long groups_per_row = k / 16;
  const long long total = rows * groups_per_row;
  uint32_t m = 0;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long g0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g0 < total; g0 += 4 * stride) {
    Raw16<T> raw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long g = g0 + u * stride;
      if (g < total) {
        const long long row = g / groups_per_row, c = (g - row * groups_per_row) * 16;
        raw[u].load(x + row * ldx + c);
      } else {
        raw[u].zero();
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float v[16];
      raw[u].to_float(v);
      m = max(m, absmax_bits16(v));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ uint32_t wm[8];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < 8; ++i) m = max(m, wm[i]);
    atomicMax(reinterpret_cast<unsigned int*>(out), m);
  }
}

__global__ void scale_pack_kernel(const unsigned char* __restrict__ s2d, long long mn, long long sf_k,
                                  unsigned char* __restrict__ blocked, long long rk, long long total) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    // i indexes the blocked buffer: (rm, rk, 32 [m%32], 4 [(m/32)%4], 4 [k%4])
    const long long atom = i >> 9;
    const int in = static_cast<int>(i & 511);
    const long long m = (atom / rk) * 128 + ((in >> 2) & 3) * 32 + (in >> 4);
    const long long kk = (atom % rk) * 4 + (in & 3);
    blocked[i] = (m < mn && kk < sf_k) ? s2d[m * sf_k + kk] : 0;
  }
}
__global__ void scale_unpack_kernel(const unsigned char* __restrict__ blocked, long long mn, long long sf_k,
                                    unsigned char* __restrict__ s2d, long long rk) {
  const long long total = mn * sf_k;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long m = i / sf_k, kk = i - m * sf_k;
    s2d[i] = blocked[((m / 128) * rk + kk / 4) * 512 + (m % 32) * 16 + ((m / 32) % 4) * 4 + (kk % 4)];
  }
}

}  // namespace qk

using namespace qk;

extern "C" size_t qk_scale_blocked_bytes(int format, long long rows, long long k) {
  const long long vec = format == QK_FMT_NVFP4 ? 16 : 32;
  const long long rm = (rows + 127) / 128, rk = ((k + vec - 1) / vec + 3) / 4;
  return static_cast<size_t>(rm * rk * 512);
}

extern "C" int qk_amax(const void* x, int x_dtype, long long rows, long long k, long long ldx, float* amax_out,
                       void* stream) {
  if (x == nullptr || amax_out == nullptr) return qk_fail(QK_ERR_INVALID_ARG, "qk_amax: null pointer");
  if (rows <= 0 || k <= 0) return QK_OK;
  if (k % 16 != 0) return qk_fail(QK_ERR_INVALID_ARG, "qk_amax: k must be a multiple of 16");
  const int esz = x_dtype == QK_DT_F32 ? 4 : 2;
  if (x_dtype != QK_DT_F32 && x_dtype != QK_DT_BF16)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_amax: input must be bf16 or fp32");
  if ((reinterpret_cast<uintptr_t>(x) % 16) || ((ldx * esz) % 16))
    return qk_fail(QK_ERR_INVALID_ARG, "qk_amax: x and its row pitch must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long groups = rows * (k / 16);
  const int blocks = static_cast<int>(std::min<long long>((groups + 1023) / 1024, 148LL * 8));
  if (x_dtype == QK_DT_BF16)
    amax_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx, rows, k, amax_out);
  else
    amax_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(x), ldx, rows, k, amax_out);
  qk_count_launch();
  return qk_check_launch("qk_amax");
}

extern "C" int qk_quantize_blockscaled_mode(int format, int scaling_mode, const void* x, int x_dtype, long long rows,
                                            long long k, long long ldx, void* codes, long long ld_codes,
                                            void* scale_blocked, const float* per_tensor_scale, void* stream) {
  if (format != QK_FMT_MXFP8_E4M3 && format != QK_FMT_MXFP8_E5M2 && format != QK_FMT_MXFP4 && format != QK_FMT_NVFP4)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_quantize_blockscaled: format must be MXFP8_E4M3, MXFP8_E5M2, MXFP4 or NVFP4");
  if (scaling_mode != QK_SCALING_DEFAULT && scaling_mode != QK_SCALING_FLOOR && scaling_mode != QK_SCALING_RCEIL)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: unknown scaling mode %d", scaling_mode);
  const bool mxfp8 = format == QK_FMT_MXFP8_E4M3 || format == QK_FMT_MXFP8_E5M2;
  if (format == QK_FMT_NVFP4 && scaling_mode != QK_SCALING_DEFAULT)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: NVFP4 scales are E4M3 values, not power-of-two: no scaling mode");
  if (format == QK_FMT_MXFP4 && scaling_mode == QK_SCALING_RCEIL)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_quantize_blockscaled: MXFP4 uses the floor rule only");
  const bool floor_mode = format == QK_FMT_MXFP4 || (mxfp8 && scaling_mode == QK_SCALING_FLOOR);
  if (x_dtype != QK_DT_F32 && x_dtype != QK_DT_BF16)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_quantize_blockscaled: input must be bf16 or fp32");
  if (rows < 0 || k < 0) return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: negative extent");
  if (rows == 0 || k == 0) return QK_OK;
  if (x == nullptr || codes == nullptr || scale_blocked == nullptr)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: null pointer");
  const int vec = format == QK_FMT_NVFP4 ? 16 : 32;
  if (k % vec != 0) return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: K must be divisible by the scale vector size");
  if (per_tensor_scale != nullptr && format != QK_FMT_NVFP4)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: only NVFP4 takes a per-tensor scale");
  const int esz = x_dtype == QK_DT_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(x) % 16) || ((ldx * esz) % 16))
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: x and its row pitch must be 16-byte aligned");
  const int cstore = mxfp8 ? 16 : 8;
  if ((reinterpret_cast<uintptr_t>(codes) % cstore) || (ld_codes % cstore))
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: codes and their row pitch must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(scale_blocked) % 16)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled: scale buffer must be 16-byte aligned");
  const long long rk_total = ((k / vec) + 3) / 4;
  const long long gx = (k + Q_TILE_COLS - 1) / Q_TILE_COLS, gy = (rows + Q_TILE_ROWS - 1) / Q_TILE_ROWS;
  if (gy > 65535) return qk_fail(QK_ERR_TOO_LARGE, "qk_quantize_blockscaled: more than 65535*128 rows");
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned char* c = static_cast<unsigned char*>(codes);
  unsigned char* s = static_cast<unsigned char*>(scale_blocked);
#define QK_LAUNCH_Q(T, F, FL)                                                                                   \
  quantize_blockscaled_kernel<T, F, FL><<<grid, Q_THREADS, 0, st>>>(static_cast<const T*>(x), ldx, rows, k, c, \
                                                                      ld_codes, s, rk_total, per_tensor_scale)
#define QK_LAUNCH_QT(F, FL)                              \
  do {                                                   \
    if (x_dtype == QK_DT_BF16) QK_LAUNCH_Q(__nv_bfloat16, F, FL); \
    else QK_LAUNCH_Q(float, F, FL);                      \
  } while (0)
  if (format == QK_FMT_MXFP8_E4M3) {
    if (floor_mode) QK_LAUNCH_QT(QK_FMT_MXFP8_E4M3, true);
    else QK_LAUNCH_QT(QK_FMT_MXFP8_E4M3, false);
  } else if (format == QK_FMT_MXFP8_E5M2) {
    if (floor_mode) QK_LAUNCH_QT(QK_FMT_MXFP8_E5M2, true);
    else QK_LAUNCH_QT(QK_FMT_MXFP8_E5M2, false);
  } else if (format == QK_FMT_MXFP4) {
    QK_LAUNCH_QT(QK_FMT_MXFP4, true);
  } else {
    QK_LAUNCH_QT(QK_FMT_NVFP4, false);
  }
#undef QK_LAUNCH_QT
#undef QK_LAUNCH_Q
  qk_count_launch();
  return qk_check_launch("qk_quantize_blockscaled");
}

extern "C" int qk_quantize_blockscaled(int format, const void* x, int x_dtype, long long rows, long long k,
                                       long long ldx, void* codes, long long ld_codes, void* scale_blocked,
                                       const float* per_tensor_scale, void* stream) {
  return qk_quantize_blockscaled_mode(format, QK_SCALING_DEFAULT, x, x_dtype, rows, k, ldx, codes, ld_codes, scale_blocked,
                                      per_tensor_scale, stream);
}

extern "C" int qk_quantize_blockscaled_dim0(int format, int scaling_mode, const void* x, int x_dtype, long long rows,
                                            long long cols, long long ldx, void* codes_t, long long ld_codes,
                                            void* scale_blocked, const float* per_tensor_scale, void* stream) {
  if (format != QK_FMT_MXFP8_E4M3 && format != QK_FMT_MXFP8_E5M2 && format != QK_FMT_MXFP4 && format != QK_FMT_NVFP4)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_quantize_blockscaled_dim0: format must be MXFP8_E4M3, MXFP8_E5M2, MXFP4 or NVFP4");
  if (scaling_mode != QK_SCALING_DEFAULT && scaling_mode != QK_SCALING_FLOOR && scaling_mode != QK_SCALING_RCEIL)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: unknown scaling mode %d", scaling_mode);
  const bool mxfp8 = format == QK_FMT_MXFP8_E4M3 || format == QK_FMT_MXFP8_E5M2;
  if (format == QK_FMT_NVFP4 && scaling_mode != QK_SCALING_DEFAULT)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: NVFP4 has no scaling mode");
  if (format == QK_FMT_MXFP4 && scaling_mode == QK_SCALING_RCEIL)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_quantize_blockscaled_dim0: MXFP4 uses the floor rule only");
  const bool floor_mode = format == QK_FMT_MXFP4 || (mxfp8 && scaling_mode == QK_SCALING_FLOOR);
  if (x_dtype != QK_DT_F32 && x_dtype != QK_DT_BF16)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_quantize_blockscaled_dim0: input must be bf16 or fp32");
  if (rows < 0 || cols < 0) return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: negative extent");
  if (rows == 0 || cols == 0) return QK_OK;
  if (x == nullptr || codes_t == nullptr || scale_blocked == nullptr)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: null pointer");
  if (rows % 32 != 0)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: the quantised extent (rows = %lld) must be a multiple of 32", rows);
  if (per_tensor_scale != nullptr && format != QK_FMT_NVFP4)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: only NVFP4 takes a per-tensor scale");
  const int esz = x_dtype == QK_DT_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(x) % 16) || ((ldx * esz) % 16))
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: x and its row pitch must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(codes_t) % 16) || (ld_codes % 16))
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: codes and their row pitch must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(scale_blocked) % 16)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_quantize_blockscaled_dim0: scale buffer must be 16-byte aligned");
  const int vec = format == QK_FMT_NVFP4 ? 16 : 32;
  const long long rk_total = ((rows / vec) + 3) / 4;
  const long long gx = (cols + QT_TILE - 1) / QT_TILE, gy = (rows + QT_TILE - 1) / QT_TILE;
  if (gy > 65535) return qk_fail(QK_ERR_TOO_LARGE, "qk_quantize_blockscaled_dim0: more than 65535*128 rows");
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned char* c = static_cast<unsigned char*>(codes_t);
  unsigned char* s = static_cast<unsigned char*>(scale_blocked);
  const size_t smem_bf16 = static_cast<size_t>(QT_TILE) * QtPitch<__nv_bfloat16>::value * 2 + 1024;
  const size_t smem_f32 = static_cast<size_t>(QT_TILE) * QtPitch<float>::value * 4 + 1024;
  int rc = QK_OK;
#define QK_LAUNCH_T(T, F, FL, SMEM)                                                                            \
  do {                                                                                                         \
    auto kern = quantize_blockscaled_t_kernel<T, F, FL>;                                                       \
    if ((SMEM) > 48 * 1024) {                                                                                  \
      /* more than the default dynamic shared memory: an attribute of the kernel in this device's context */   \
      static std::mutex mu;                                                                                    \
      static bool done[64] = {};                                                                               \
      int dev = -1;                                                                                            \
      cudaGetDevice(&dev);                                                                                     \
      rc = qk::set_once_per_device(mu, done, dev, [&]() -> int {                                               \
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM)); \
        return e == cudaSuccess ? QK_OK : qk_fail(QK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e)); \
      });                                                                                                      \
    }                                                                                                          \
    if (rc == QK_OK)                                                                                           \
      kern<<<grid, Q_THREADS, (SMEM), st>>>(static_cast<const T*>(x), ldx, rows, cols, c, ld_codes, s, rk_total, per_tensor_scale); \
  } while (0)
#define QK_LAUNCH_TT(F, FL)                                             \
  do {                                                                  \
    if (x_dtype == QK_DT_BF16) QK_LAUNCH_T(__nv_bfloat16, F, FL, smem_bf16); \
    else QK_LAUNCH_T(float, F, FL, smem_f32);                           \
  } while (0)
  if (format == QK_FMT_MXFP8_E4M3) {
    if (floor_mode) QK_LAUNCH_TT(QK_FMT_MXFP8_E4M3, true);
    else QK_LAUNCH_TT(QK_FMT_MXFP8_E4M3, false);
  } else if (format == QK_FMT_MXFP8_E5M2) {
    if (floor_mode) QK_LAUNCH_TT(QK_FMT_MXFP8_E5M2, true);
    else QK_LAUNCH_TT(QK_FMT_MXFP8_E5M2, false);
  } else if (format == QK_FMT_MXFP4) {
    QK_LAUNCH_TT(QK_FMT_MXFP4, true);
  } else {
    QK_LAUNCH_TT(QK_FMT_NVFP4, false);
  }
#undef QK_LAUNCH_TT
#undef QK_LAUNCH_T
  if (rc != QK_OK) return rc;
  qk_count_launch();
  return qk_check_launch("qk_quantize_blockscaled_dim0");
}

extern "C" int qk_scale_pack_blocked(const void* scale_2d, long long mn, long long sf_k, void* blocked, void* stream) {
  if (mn <= 0 || sf_k <= 0) return QK_OK;
  if (scale_2d == nullptr || blocked == nullptr) return qk_fail(QK_ERR_INVALID_ARG, "qk_scale_pack_blocked: null pointer");
  const long long rm = (mn + 127) / 128, rk = (sf_k + 3) / 4, total = rm * rk * 512;
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 32));
  scale_pack_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const unsigned char*>(scale_2d), mn, sf_k, static_cast<unsigned char*>(blocked), rk, total);
  qk_count_launch();
  return qk_check_launch("qk_scale_pack_blocked");
}

extern "C" int qk_scale_unpack_blocked(const void* blocked, long long mn, long long sf_k, void* scale_2d, void* stream) {
  if (mn <= 0 || sf_k <= 0) return QK_OK;
  if (scale_2d == nullptr || blocked == nullptr) return qk_fail(QK_ERR_INVALID_ARG, "qk_scale_unpack_blocked: null pointer");
  const long long rk = (sf_k + 3) / 4, total = mn * sf_k;
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 32));
  scale_unpack_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const unsigned char*>(blocked), mn, sf_k, static_cast<unsigned char*>(scale_2d), rk);
  qk_count_launch();
  return qk_check_launch("qk_scale_unpack_blocked");
}
