// Row-wise normalisation kernels of the DiT block (sm_100a).
//
//   adaln_rmsnorm   out = RMSNorm(x) * w * (1 + table[idx[r], scale]) + table[idx[r], shift]
//                   (reference src/models/ops/fused_block.py:41-44, fused: one read of x,
//                   one write, the per-row AdaLN gather done in registers)
//   frame_sums      per-frame column sums of the video rows (fp32), for the linear branch's
//                   alpha (reference linear_attention/branch.py:440-442)
//   qk_prep         per-head RMSNorm then rotate-half RoPE (softmax_attention/kernels.py:27-30)
#include "common.cuh"
#include "launchers.h"

namespace vdn {

// One warp per row; VPL 16-byte vectors per lane held in registers.
template <int VPL>
__global__ void __launch_bounds__(256) adaln_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const float* __restrict__ w, float eps,
    const __nv_bfloat16* __restrict__ table, int64_t ldt, int shift_col, int scale_col,
    const int* __restrict__ idx, NormDst dst, int T, int D) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int nvec = D >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * ldx);
  uint4 v[VPL];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      v[i] = xr[c];
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a = bf16_lo(u[j]), b = bf16_hi(u[j]);
        ss += a * a + b * b;
      }
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)D + eps);
  const int ti = idx[row];
  const __nv_bfloat16* trow = table + (int64_t)ti * ldt;
  const int64_t drow = dst.row0 + row;   // row in the destination buffers
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
      const uint4 sh = *reinterpret_cast<const uint4*>(trow + shift_col + c * 8);
      const uint4 sc = *reinterpret_cast<const uint4*>(trow + scale_col + c * 8);
      const uint32_t* shu = reinterpret_cast<const uint32_t*>(&sh);
      const uint32_t* scu = reinterpret_cast<const uint32_t*>(&sc);
      uint32_t res[4];
      float wv[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      if (w) {
        const float4 wa = __ldg(reinterpret_cast<const float4*>(w + c * 8));
        const float4 wb = __ldg(reinterpret_cast<const float4*>(w + c * 8 + 4));
        wv[0] = wa.x; wv[1] = wa.y; wv[2] = wa.z; wv[3] = wa.w;
        wv[4] = wb.x; wv[5] = wb.y; wv[6] = wb.z; wv[7] = wb.w;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a = bf16_lo(u[j]) * rstd * wv[2 * j], b = bf16_hi(u[j]) * rstd * wv[2 * j + 1];
        a = a * (1.f + bf16_lo(scu[j])) + bf16_lo(shu[j]);
        b = b * (1.f + bf16_hi(scu[j])) + bf16_hi(shu[j]);
        res[j] = pack_bf16(a, b);
      }
#pragma unroll
      for (int d = 0; d < 2; ++d)
        if (dst.out[d])
          reinterpret_cast<uint4*>(dst.out[d] + drow * dst.ldo)[c] =
              make_uint4(res[0], res[1], res[2], res[3]);
      if (dst.q[0]) {
        // E4M3 copy for an fp8 GEMM: a half-warp holds one 1x128 block (D % 256 == 0, so
        // every lane of the warp is here); the bf16-rounded values are quantised
        float f[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          f[2 * j] = bf16_lo(res[j]);
          f[2 * j + 1] = bf16_hi(res[j]);
        }
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const int e = e8_exponent(amax);
        const float inv = exp2_int(-e < -126 ? -126 : (-e > 127 ? 127 : -e));
        const uint32_t lo = (uint32_t)pack_e4m3x2(f[0] * inv, f[1] * inv) |
                            ((uint32_t)pack_e4m3x2(f[2] * inv, f[3] * inv) << 16);
        const uint32_t hi = (uint32_t)pack_e4m3x2(f[4] * inv, f[5] * inv) |
                            ((uint32_t)pack_e4m3x2(f[6] * inv, f[7] * inv) << 16);
        const uint32_t bb = (uint32_t)(e + 127) & 0xFF;
#pragma unroll
        for (int d = 0; d < 2; ++d) {
          if (!dst.q[d]) continue;
          *reinterpret_cast<uint2*>(dst.q[d] + drow * dst.ldq + c * 8) = make_uint2(lo, hi);
          if ((lane & 15) == 0)
            *reinterpret_cast<uint32_t*>(dst.qsf[d] + sf_offset(drow, (int64_t)(c / 16) * 4, D / 32)) =
                bb | (bb << 8) | (bb << 16) | (bb << 24);
        }
      }
    }
  }
}

void launch_adaln_rmsnorm(const void* x, int64_t ldx, const float* w, float eps, const void* table,
                          int64_t ldt, int shift_col, int scale_col, const int* idx, void* out,
                          int64_t ldo, int T, int D, cudaStream_t stream, void* q, int64_t ldq,
                          void* qsf) {
  NormDst dst{};
  dst.out[0] = reinterpret_cast<__nv_bfloat16*>(out);
  dst.ldo = ldo;
  dst.q[0] = reinterpret_cast<uint8_t*>(q);
  dst.qsf[0] = reinterpret_cast<uint8_t*>(qsf);
  dst.ldq = ldq;
  launch_adaln_rmsnorm_dst(x, ldx, w, eps, table, ldt, shift_col, scale_col, idx, dst, T, D, stream);
}

void launch_adaln_rmsnorm_dst(const void* x, int64_t ldx, const float* w, float eps,
                              const void* table, int64_t ldt, int shift_col, int scale_col,
                              const int* idx, const NormDst& dst, int T, int D,
                              cudaStream_t stream) {
  if (T == 0) return;
  const int nvec = D / 8;
  const int need = (nvec + 31) / 32;
  dim3 grid((T + 7) / 8), block(256);
  auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto tb = reinterpret_cast<const __nv_bfloat16*>(table);
#define VDN_ADALN(N)                                                                          \
  adaln_rmsnorm_kernel<N><<<grid, block, 0, stream>>>(xb, ldx, w, eps, tb, ldt, shift_col,    \
                                                       scale_col, idx, dst, T, D)
  if (need <= 1) VDN_ADALN(1);
  else if (need <= 2) VDN_ADALN(2);
  else if (need <= 4) VDN_ADALN(4);
  else if (need <= 8) VDN_ADALN(8);
  else if (need <= 16) VDN_ADALN(16);
  else if (need <= 24) VDN_ADALN(24);
  else VDN_ADALN(48);
#undef VDN_ADALN
}

// Column sums of video rows grouped by frame: out[f, c] = sum over the rows of frame f that
// lie in x (x[0] is packed row `row0`, x holds `nrows` rows; frame f is packed rows
// [vs + f*S, vs + (f+1)*S)). grid (F, ceil(D/256)); lane = 8 columns, warps stride rows.
// With dst.n > 0 the partial sums go to dst.n destinations instead of `out` (the peers'
// slots in symmetric memory, plain stores over NVLink): frame f's sums land at
// dst.base[p] + dst.offset + f * D, and only frames this shard touches are stored -- the
// slots of the others stay at the zero they were cleared to, so a receiver may sum all slots.
__global__ void __launch_bounds__(256) frame_sums_kernel(const __nv_bfloat16* __restrict__ x,
                                                         int64_t ldx, int64_t row0, int64_t nrows,
                                                         int64_t vs, int S, int D,
                                                         float* __restrict__ out, FrameSumDst dst) {
  __shared__ float red[8][256];
  const int f = blockIdx.x;
  const int c0 = blockIdx.y * 256;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = c0 + lane * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int64_t a = max(vs + (int64_t)f * S, row0) - row0;
  const int64_t b = min(vs + (int64_t)(f + 1) * S, row0 + nrows) - row0;
  if (col < D) {
    for (int64_t s = a + warp; s < b; s += 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + s * ldx + col);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += bf16_lo(u[j]);
        acc[2 * j + 1] += bf16_hi(u[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = acc[j];
  __syncthreads();
  const int t = threadIdx.x;
  if (c0 + t < D) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][t];
    if (dst.n == 0) {
      out[(int64_t)f * D + c0 + t] = s;
    } else if (b > a) {
      for (int p = 0; p < dst.n; ++p) dst.base[p][dst.offset + (int64_t)f * D + c0 + t] = s;
    }
  }
}

void launch_frame_sums(const void* x, int64_t ldx, int64_t row0, int64_t nrows, int64_t vs,
                       int F, int S, int D, float* out, cudaStream_t stream,
                       const FrameSumDst* dst) {
  if (F == 0) return;
  dim3 grid(F, (D + 255) / 256);
  FrameSumDst d{};
  if (dst) d = *dst;
  frame_sums_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                              row0, nrows, vs, S, D, out, d);
}

// One warp per (row, head). Generic head_dim <= 256 (multiple of 2), rotary_dim <= head_dim.
__global__ void __launch_bounds__(256) qk_prep_kernel(
    const __nv_bfloat16* __restrict__ src, int64_t lds, int T, int H, int d,
    const float* __restrict__ w, float eps, const float* __restrict__ cosv,
    const float* __restrict__ sinv, int rot, __nv_bfloat16* __restrict__ out, int64_t ldo) {
  __shared__ float buf[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * 8 + warp;
  if (item >= (int64_t)T * H) return;
  const int row = (int)(item / H), h = (int)(item % H);
  const __nv_bfloat16* s = src + (int64_t)row * lds + h * d;
  float* b = buf[warp];
  float ss = 0.f;
  for (int i = lane * 2; i < d; i += 64) {
    const __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162*>(s + i);
    const float a = __bfloat162float(p.x), c = __bfloat162float(p.y);
    b[i] = a;
    b[i + 1] = c;
    ss += a * a + c * c;
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)d + eps);
  for (int i = lane * 2; i < d; i += 64) {
    b[i] *= rstd * w[i];
    b[i + 1] *= rstd * w[i + 1];
  }
  __syncwarp();
  const float* cr = cosv + (int64_t)row * rot;
  const float* sr = sinv + (int64_t)row * rot;
  const int half = rot >> 1;
  __nv_bfloat16* o = out + (int64_t)row * ldo + h * d;
  for (int i = lane * 2; i < d; i += 64) {
    float r[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int e = i + j;
      if (e < rot) {
        const float rotated = e < half ? -b[e + half] : b[e - half];
        r[j] = b[e] * cr[e] + rotated * sr[e];
      } else {
        r[j] = b[e];
      }
    }
    *reinterpret_cast<__nv_bfloat162*>(o + i) = __floats2bfloat162_rn(r[0], r[1]);
  }
}

void launch_qk_prep(const void* src, int64_t lds, int T, int H, int d, const float* w, float eps,
                    const float* cosv, const float* sinv, int rot, void* out, int64_t ldo,
                    cudaStream_t stream) {
  const int64_t items = (int64_t)T * H;
  if (items == 0) return;
  qk_prep_kernel<<<(unsigned)((items + 7) / 8), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(src), lds, T, H, d, w, eps, cosv, sinv, rot,
      reinterpret_cast<__nv_bfloat16*>(out), ldo);
}

// Tensor-parallel residual: x += gate[idx[r]] * (a + b + bias), a and b the two ranks'
// bf16 partial sums of a row-parallel GEMM for this rank's rows (added in fp32). One warp
// per row, 8 columns per lane per step.
__global__ void __launch_bounds__(256) residual_combine_kernel(
    __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ a,
    const __nv_bfloat16* __restrict__ b, int64_t ldp, const float* __restrict__ bias,
    const __nv_bfloat16* __restrict__ gate, int64_t ldg, const int* __restrict__ idx, int R,
    int D) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const __nv_bfloat16* g = gate + (int64_t)idx[row] * ldg;
  for (int c = lane * 8; c < D; c += 256) {
    const uint4 av = *reinterpret_cast<const uint4*>(a + (int64_t)row * ldp + c);
    const uint4 bv = *reinterpret_cast<const uint4*>(b + (int64_t)row * ldp + c);
    const uint32_t* aw = reinterpret_cast<const uint32_t*>(&av);
    const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bv);
    float y[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      y[2 * j] = bf16_lo(aw[j]) + bf16_lo(bw[j]);
      y[2 * j + 1] = bf16_hi(aw[j]) + bf16_hi(bw[j]);
    }
    if (bias) {
      const float4 c0 = *reinterpret_cast<const float4*>(bias + c);
      const float4 c1 = *reinterpret_cast<const float4*>(bias + c + 4);
      y[0] += c0.x; y[1] += c0.y; y[2] += c0.z; y[3] += c0.w;
      y[4] += c1.x; y[5] += c1.y; y[6] += c1.z; y[7] += c1.w;
    }
    uint4 xv = *reinterpret_cast<const uint4*>(x + (int64_t)row * ldx + c);
    const uint4 gv = *reinterpret_cast<const uint4*>(g + c);
    uint32_t* xw = reinterpret_cast<uint32_t*>(&xv);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      xw[j] = pack_bf16(bf16_lo(xw[j]) + bf16_lo(gw[j]) * y[2 * j],
                        bf16_hi(xw[j]) + bf16_hi(gw[j]) * y[2 * j + 1]);
    *reinterpret_cast<uint4*>(x + (int64_t)row * ldx + c) = xv;
  }
}

void launch_residual_combine(void* x, int64_t ldx, const void* a, const void* b, int64_t ldp,
                             const float* bias, const void* gate, int64_t ldg, const int* idx,
                             int R, int D, cudaStream_t stream) {
  if (R == 0) return;
  residual_combine_kernel<<<(R + 7) / 8, 256, 0, stream>>>(
      reinterpret_cast<__nv_bfloat16*>(x), ldx, reinterpret_cast<const __nv_bfloat16*>(a),
      reinterpret_cast<const __nv_bfloat16*>(b), ldp, bias,
      reinterpret_cast<const __nv_bfloat16*>(gate), ldg, idx, R, D);
}

}  // namespace vdn
