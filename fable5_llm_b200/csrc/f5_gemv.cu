// Batch-1 W4A8 GEMV over the reference's packed DDR row format (sm_100a).
//
// Law (ref/w4a8_ref.py:254-289 matvec_y32):
//   acc_g = sum_{k in group g} w4[k] * x8[k]      (int32)
//   p     = sum_g m_g * acc_g                      (int64, < 2^41)
//   y32   = rshift_round(p, sh)
// followed by a fused epilogue (ref/layer_fixed.py:1224-1236 matvec_to's
// second shift, clip16, residual add, the MLP silu*up product of
// ref/layer_fixed.py:1597-1604, or the LM-head running argmax of
// ref/gen_model_script.py:641).
//
// Memory layout: the weights stay in the reference's own row format
// (ref/w4a8_ref.py:102-114: K/128 64-byte weight beats, low nibble = even k,
// then ceil(NG/32) beats of little-endian uint16 group mantissas), i.e.
// exactly 4.125 bits/weight, 64-byte aligned rows.  A row is streamed by one
// warp with 16-byte non-allocating loads: lane l of chunk c reads bytes
// [c*512 + 16l, +16) = weights k in [c*1024 + 32l, +32).  A 16-byte load
// never straddles a group (g = 128 or 64).
//
// Nibble arithmetic: (word << 4) & 0xF0F0F0F0 puts each even-k nibble in the
// high half of its byte, which read as int8 is 16*w; word & 0xF0F0F0F0 does
// the same for odd k.  Two dp4a against the even/odd-permuted x8 bytes give
// 16*sum(w*x) exactly; the factor 16 is removed once per row (p16 >> 4 is
// exact because every term is a multiple of 16).  The int64 group-scale FMA
// m_g * acc is applied per lane-chunk (linear, so summing partial group sums
// times m_g equals m_g times the group sum -- integer arithmetic is exact
// and order-free).
#include "f5_int.cuh"
#include "f5_kernels.cuh"

namespace f5 {

F5_DEV uint4 ld_stream16(const uint8_t *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
F5_DEV uint32_t ld_u16(const uint8_t *p) {
  unsigned short v;
  asm("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

F5_DEV int dot_word(uint32_t w, uint2 x, int acc) {
  acc = __dp4a((int)((w << 4) & 0xF0F0F0F0u), (int)x.x, acc);
  acc = __dp4a((int)(w & 0xF0F0F0F0u), (int)x.y, acc);
  return acc;
}
F5_DEV int dot32(uint4 w, uint2 x0, uint2 x1, uint2 x2, uint2 x3) {
  int acc = dot_word(w.x, x0, 0);
  acc = dot_word(w.y, x1, acc);
  acc = dot_word(w.z, x2, acc);
  acc = dot_word(w.w, x3, acc);
  return acc;   // 16 * sum(w*x) over 32 weights, |.| < 2^20
}

F5_DEV unsigned long long argmax_key(int32_t y, int row) {
  return ((unsigned long long)((uint32_t)y ^ 0x80000000u) << 32) |
         (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}

// y32 for one row from the lane-reduced p16 (= 16 p)
F5_DEV int32_t finish_y32(long long p16, int sh, uint32_t *err, long long *p_exact) {
  const long long p = p16 >> 4;
  const long long y = rshr(p, sh);
  if (y >= (1ll << 31) || y <= -(1ll << 31)) atomicOr(err, DERR_Y32_OVERFLOW);
  if (p_exact) *p_exact = p;
  return (int32_t)y;
}

template <int NCH>
__global__ void __launch_bounds__(256, 2) k_gemv(const __grid_constant__ GemvArgs a) {
  extern __shared__ uint2 xs[];
  const int tid = threadIdx.x, lane = tid & 31;
  const int wpb = blockDim.x >> 5;
  const int nw = gridDim.x * wpb;
  const int gw = blockIdx.x * wpb + (tid >> 5);
  const int K2 = a.K >> 1;
  const int gshift = (a.g == 128) ? 6 : 5;

  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // x8 -> lane-major even/odd layout: 8-k block b sits at [(c*4 + j)*32 + l]
  const int nblk = a.K >> 3;
  for (int b = tid; b < nblk; b += blockDim.x) {
    const uint2 v = *reinterpret_cast<const uint2 *>(a.x8 + 8 * b);
    uint2 o;
    o.x = __byte_perm(v.x, v.y, 0x6420);
    o.y = __byte_perm(v.x, v.y, 0x7531);
    xs[(((b >> 7) << 2) + (b & 3)) * 32 + ((b >> 2) & 31)] = o;
  }
  int e_x = 0, in_f = 0;
  if (a.xmeta) { e_x = a.xmeta[0]; in_f = a.xmeta[1]; }
  __syncthreads();

  unsigned long long best = 0ull;
  for (int u = gw; u < a.total_units; u += nw) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < GEMV_MAX_SEG; ++i)
      if (i < a.nseg && u >= a.seg[i].unit_begin) s = i;
    const GemvSeg &sg = a.seg[s];
    const int ul = u - sg.unit_begin;
    const bool paired = sg.mode == GM_SILU_MUL;
    int rA, rB;
    const uint8_t *pa, *pb;
    bool vB;
    if (paired) {
      rA = rB = ul;
      pa = sg.w + (size_t)ul * a.stride;
      pb = sg.w2 + (size_t)ul * a.stride;
      vB = true;
    } else {
      rA = 2 * ul;
      rB = rA + 1;
      vB = rB < sg.rows;
      pa = sg.w + (size_t)rA * a.stride;
      pb = vB ? pa + a.stride : pa;
    }
    long long accA = 0, accB = 0;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int boff = c * 512 + lane * 16;
      if (boff < K2) {
        const uint4 wa = ld_stream16(pa + boff);
        const uint4 wb = ld_stream16(pb + boff);
        const int moff = K2 + 2 * (boff >> gshift);
        const uint32_t ma = ld_u16(pa + moff);
        const uint32_t mb = ld_u16(pb + moff);
        const uint2 *xr = xs + (c << 2) * 32 + lane;
        const uint2 x0 = xr[0], x1 = xr[32], x2 = xr[64], x3 = xr[96];
        accA += (long long)ma * dot32(wa, x0, x1, x2, x3);
        accB += (long long)mb * dot32(wb, x0, x1, x2, x3);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      accA += __shfl_xor_sync(0xffffffffu, accA, o);
      accB += __shfl_xor_sync(0xffffffffu, accB, o);
    }
    if (sg.mode == GM_ARGMAX) {
      if (lane == 0) {
        const int32_t ya = finish_y32(accA, a.sh, a.err, nullptr);
        unsigned long long k = argmax_key(ya, sg.out_row0 + rA);
        if (vB) {
          const int32_t yb = finish_y32(accB, a.sh, a.err, nullptr);
          const unsigned long long kb = argmax_key(yb, sg.out_row0 + rB);
          k = kb > k ? kb : k;
        }
        best = k > best ? k : best;
      }
      continue;
    }
    if (paired) {
      if (lane == 0) {
        const int32_t yg = finish_y32(accA, a.sh, a.err, nullptr);
        const int32_t yu = finish_y32(accB, a.sh, a.err, nullptr);
        const int64_t gq = shift_to(yg, (15 - sg.e - a.sh) - e_x + in_f - sg.out_f);
        const int64_t uq = shift_to(yu, (15 - sg.e2 - a.sh) - e_x + in_f - sg.out_f2);
        const int64_t sgv = clip16(silu_q(clip(gq, -(1 << 20), (1 << 20) - 1)));
        static_cast<int16_t *>(sg.out)[sg.out_row0 + rA] = (int16_t)clip16(rshr(sgv * uq, 12));
      }
      continue;
    }
    if (lane < 2 && (lane == 0 || vB)) {
      const int row = lane == 0 ? rA : rB;
      long long pex;
      const int32_t y = finish_y32(lane == 0 ? accA : accB, a.sh, a.err, &pex);
      const int orow = sg.out_row0 + row;
      if (sg.p_out) sg.p_out[orow] = pex;
      const int sh2 = (15 - sg.e - a.sh) - e_x + in_f - sg.out_f;
      switch (sg.mode) {
        case GM_Y32: static_cast<int32_t *>(sg.out)[orow] = y; break;
        case GM_TO16: static_cast<int16_t *>(sg.out)[orow] = (int16_t)clip16(shift_to(y, sh2)); break;
        case GM_TO64: static_cast<int64_t *>(sg.out)[orow] = shift_to(y, sh2); break;
        case GM_RESID: {
          int16_t *o = static_cast<int16_t *>(sg.out) + orow;
          *o = (int16_t)clip16((int64_t)*o + clip16(shift_to(y, sh2)));
        } break;
        default: break;
      }
    }
  }
  if (a.argmax_key) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if (lane == 0 && best) atomicMax(a.argmax_key, best);
  }
}

template <int NCH>
static cudaError_t launch_nch(const GemvArgs &a, cudaStream_t st, bool pdl, int max_blocks) {
  const int threads = 256;
  int blocks = (a.total_units + 7) / 8;
  if (blocks > max_blocks) blocks = max_blocks;
  if (blocks < 1) blocks = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = NCH * 4 * 32 * sizeof(uint2);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_gemv<NCH>, a);
}

cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t st, bool pdl, int max_blocks) {
  const int nch = (a.K + 1023) / 1024;
  switch (nch) {
    case 1: return launch_nch<1>(a, st, pdl, max_blocks);
    case 2: return launch_nch<2>(a, st, pdl, max_blocks);
    case 3: return launch_nch<3>(a, st, pdl, max_blocks);
    case 4: return launch_nch<4>(a, st, pdl, max_blocks);
    case 5: return launch_nch<5>(a, st, pdl, max_blocks);
    case 6: return launch_nch<6>(a, st, pdl, max_blocks);
    case 7: return launch_nch<7>(a, st, pdl, max_blocks);
    case 8: return launch_nch<8>(a, st, pdl, max_blocks);
    case 9: return launch_nch<9>(a, st, pdl, max_blocks);
    case 10: return launch_nch<10>(a, st, pdl, max_blocks);
    case 11: return launch_nch<11>(a, st, pdl, max_blocks);
    case 12: return launch_nch<12>(a, st, pdl, max_blocks);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace f5
