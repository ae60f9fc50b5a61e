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
#include "f5_gemv_core.cuh"

namespace f5 {

constexpr int GT_CONS = 16;                     // consumer warps
constexpr int GT_CTHREADS = GT_CONS * 32;
constexpr int GT_THREADS = GT_CTHREADS + 32;    // + one producer warp
constexpr int GT_MAX_STAGES = 4;
constexpr int GT_CTA_SMEM = 232448 - 6144;      // dynamic smem per CTA (one CTA per SM)
constexpr int GT_RES_MAX = 2048;                // deferred row results per CTA
constexpr unsigned long long GT_WAIT_NS = 2000000000ull;   // 2 s: a safety net only

// Persistent TMA-pipelined GEMV: a producer warp streams contiguous blocks
// of packed rows (cp.async.bulk, 16-byte aligned, single destination) into
// shared-memory stages guarded by full/empty mbarriers; sixteen consumer
// warps reduce one row per warp out of shared memory, park the row's p16 in
// shared memory and release the stage at once.  The per-row epilogues run
// after the CTA's last chunk with every consumer thread taking one row, so
// the serial int64 epilogue never sits on the weight-stream critical path.
// The first stages are issued BEFORE griddepcontrol.wait: the weights do not
// depend on the previous kernel, so under programmatic dependent launch the
// weight stream overlaps the producer kernel's tail.
template <int NCH>
__global__ void __launch_bounds__(GT_THREADS, 1) k_gemv(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar_full[GT_MAX_STAGES], bar_empty[GT_MAX_STAGES];
  __shared__ long long red[32];
  __shared__ long long s_r;
  __shared__ int s_meta[4];
  __shared__ volatile int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K2 = a.K >> 1;
  const int gshift = (a.g == 128) ? 6 : 5;
  const int NS = a.stages;
  const uint32_t stage_bytes = (uint32_t)a.rows_per_stage * (uint32_t)a.stride;
  uint2 *xs = reinterpret_cast<uint2 *>(smem + NS * stage_bytes);
  long long *s_res = reinterpret_cast<long long *>(smem + NS * stage_bytes + NCH * 4 * 32 * sizeof(uint2));
  const int G = gridDim.x, b = blockIdx.x;
  const int u0 = (int)((long long)a.total_units * b / G);
  const int u1 = (int)((long long)a.total_units * (b + 1) / G);

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], GT_CONS);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // producer: the first NS chunks need no empty-wait -> issue them now
  int pu = u0, pi = 0;
  if (warp == GT_CONS && lane == 0) {
    Chunk ch;
    while (pi < NS && next_chunk(a, pu, u1, ch)) {
      const GemvSeg &sg = a.seg[ch.seg];
      const uint32_t nb = (uint32_t)ch.n * a.stride;
      uint8_t *dst = smem + pi * stage_bytes;
      const bool pair = sg.mode == GM_SILU_MUL;
      mbar_expect_tx(&bar_full[pi], pair ? 2 * nb : nb);
      bulk_g2s_stream(dst, sg.w + (size_t)ch.r0 * a.stride, nb, &bar_full[pi]);
      if (pair) bulk_g2s_stream(dst + nb, sg.w2 + (size_t)ch.r0 * a.stride, nb, &bar_full[pi]);
      ++pi;
    }
  }

  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- prologue (all warps): x8 into the lane-major even/odd layout ----
  const int nblk = a.K >> 3;
  if (a.pro.mode == PRO_X8) {
    for (int bb = tid; bb < nblk; bb += blockDim.x) {
      const uint2 v = *reinterpret_cast<const uint2 *>(a.x8 + 8 * bb);
      uint2 o;
      o.x = __byte_perm(v.x, v.y, 0x6420);
      o.y = __byte_perm(v.x, v.y, 0x7531);
      xs[(((bb >> 7) << 2) + (bb & 3)) * 32 + ((bb >> 2) & 31)] = o;
    }
    if (tid == 0) {
      s_meta[0] = a.xmeta ? a.xmeta[0] : 0;
      s_meta[1] = a.xmeta ? a.xmeta[1] : 0;
    }
  } else {
    prologue<(NCH * 128 + GT_THREADS - 1) / GT_THREADS>(BlockSync(), a, xs, red, &s_r, s_meta);
  }
  __syncthreads();
  const int e_x = s_meta[0], in_f = s_meta[1];

  if (warp == GT_CONS) {
    // ---- producer: remaining chunks, each after its stage is released ----
    if (lane == 0) {
      Chunk ch;
      int issued = pi;
      while (!s_abort && next_chunk(a, pu, u1, ch)) {
        const int s = issued % NS;
        if (!mbar_wait(&bar_empty[s], ((issued / NS) - 1) & 1, GT_WAIT_NS)) {
          s_abort = 1;
          atomicOr(a.err, DERR_TIMEOUT);
          break;
        }
        const GemvSeg &sg = a.seg[ch.seg];
        const uint32_t nb = (uint32_t)ch.n * a.stride;
        uint8_t *dst = smem + s * stage_bytes;
        const bool pair = sg.mode == GM_SILU_MUL;
        mbar_expect_tx(&bar_full[s], pair ? 2 * nb : nb);
        bulk_g2s_stream(dst, sg.w + (size_t)ch.r0 * a.stride, nb, &bar_full[s]);
        if (pair) bulk_g2s_stream(dst + nb, sg.w2 + (size_t)ch.r0 * a.stride, nb, &bar_full[s]);
        ++issued;
      }
      // never leave the CTA with copies in flight: drain every issued stage
      // the consumers have not waited on (bounded)
      if (s_abort) {
        for (int i = max(0, issued - NS); i < issued; ++i)
          mbar_wait(&bar_full[i % NS], (i / NS) & 1, GT_WAIT_NS);
      }
    }
    return;
  }

  // ---- consumers: one row per warp, results parked in s_res ----
  uint2 xr[4][4];
  if (NCH <= 4) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) xr[c][j] = c < NCH ? xs[((c << 2) + j) * 32 + lane] : make_uint2(0, 0);
  }
  int cu = u0, ci = 0;
  Chunk ch;
  while (next_chunk(a, cu, u1, ch)) {
    const int s = ci % NS;
    if (s_abort || !mbar_wait(&bar_full[s], (ci / NS) & 1, GT_WAIT_NS)) {
      if (!s_abort) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
      break;
    }
    const uint8_t *st = smem + s * stage_bytes;
    const bool pair = a.seg[ch.seg].mode == GM_SILU_MUL;
    const int nrows = pair ? 2 * ch.n : ch.n;
    const int cbase = ch.u - u0;
    for (int r = warp; r < nrows; r += GT_CONS) {
      const long long aa = warp_sum_row(row_dot<NCH>(st + (size_t)r * a.stride, K2, gshift, lane, xr, xs));
      if (lane == 0) s_res[pair ? (r < ch.n ? 2 * (cbase + r) : 2 * (cbase + r - ch.n) + 1) : cbase + r] = aa;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar_empty[s]);
    ++ci;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(GT_CTHREADS) : "memory");
  if (s_abort) return;

  // ---- deferred epilogues: one unit per consumer thread ----
  unsigned long long best = 0ull;
  RStat rs;
  for (int i = tid; i < u1 - u0; i += GT_CTHREADS) {
    const int u = u0 + i;
    const GemvSeg &sg = a.seg[seg_of(a, u)];
    const int row = u - sg.unit_begin;
    if (sg.mode == GM_SILU_MUL) {
      epilogue_pair(a, sg, row, s_res[2 * i], s_res[2 * i + 1], e_x, in_f);
    } else {
      epilogue_row(a, sg, row, s_res[i], e_x, in_f, best, 0, sg.rstat ? &rs : nullptr);
    }
  }
  if (a.nseg == 1 && a.seg[0].rstat) rstat_flush(a.seg[0].rstat, rs);
  if (a.argmax_key) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if (lane == 0 && best) atomicMax(a.argmax_key, best);
  }
}

int gemv_rows_per_stage(int stride) {
  int r = 53248 / stride;     // <= 52 KB stages: 16 rows at K=4096, 8 at K=12288
  if (r > 16) r = 16;
  if (r < 2) r = 2;
  return r;
}

template <int NCH>
static cudaError_t launch_nch(GemvArgs a, cudaStream_t st, bool pdl, int max_blocks) {
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv<NCH>, cudaFuncAttributeMaxDynamicSharedMemorySize, GT_CTA_SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int ru = a.rows_per_stage;
  int blocks = (a.total_units + ru - 1) / ru;
  if (blocks > max_blocks) blocks = max_blocks;
  const int min_blocks = (a.total_units + GT_RES_MAX - 1) / GT_RES_MAX;
  if (blocks < min_blocks) blocks = min_blocks;
  if (blocks < 1) blocks = 1;
  bool paired = false;
  for (int i = 0; i < a.nseg; ++i) paired |= a.seg[i].mode == GM_SILU_MUL;
  const size_t per_cta = (size_t)(a.total_units + blocks - 1) / blocks + 1;
  const size_t res_bytes = per_cta * (paired ? 2 : 1) * sizeof(long long);
  const size_t xs_bytes = (size_t)NCH * 4 * 32 * sizeof(uint2);
  const size_t stage_bytes = (size_t)a.rows_per_stage * a.stride;
  int stages = (int)(((long long)GT_CTA_SMEM - (long long)xs_bytes - (long long)res_bytes) / (long long)stage_bytes);
  if (stages > GT_MAX_STAGES) stages = GT_MAX_STAGES;
  if (stages < 2) return cudaErrorInvalidValue;
  a.stages = stages;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(GT_THREADS);
  cfg.dynamicSmemBytes = stages * stage_bytes + xs_bytes + res_bytes;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_gemv<NCH>, a);
}

cudaError_t launch_gemv(const GemvArgs &a_in, cudaStream_t st, bool pdl, int max_blocks) {
  GemvArgs a = a_in;
  a.rows_per_stage = gemv_rows_per_stage(a.stride);
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
