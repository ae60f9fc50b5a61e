// Batched W4A8 decode GEMM on the 5th-generation tensor cores (sm_100a).
//
// B independent sequences share one weight image, so every projection of
// the decode step becomes Y[b][row] = matvec_y32(w4, m, sh, x8[b])
// (ref/w4a8_ref.py:254-289) for b < B:
//   acc_g[row][b] = sum_{k in g} w4[row][k] * x8[b][k]       (int32, |.| <= 2^17)
//   p[row][b]     = sum_g m_g[row] * acc_g[row][b]            (int64)
//   y32           = rshift_round(p, sh)
// acc_g is a 128 x Bp x 128 int8 matrix product per group: tcgen05.mma
// kind::i8 with an int32 accumulator in tensor memory (TMEM), one MMA tile
// of 128 weight rows x Bp sequences per group.  The group scale is applied
// by the epilogue warps, which read each group's accumulator out of TMEM and
// fold m_g * acc_g into int64 registers (a different m_g per row and group
// rules out accumulating across groups inside the MMA).
//
// The weights stay in the reference's packed row format in HBM.  A stage
// brings 4 groups (256 bytes) of each of the tile's 128 rows into shared
// memory with one 2D tensor-map copy.  The nibbles become 16 * w4 as signed
// bytes with one shift and two masks per 8 weights ((word << 4) & 0xF0F0F0F0
// for even k, word & 0xF0F0F0F0 for odd k), written in the MMA's
// 128-byte-swizzled K-major layout; the accumulator then holds 16 * acc_g
// (|.| <= 2^21) and p = (sum_g m_g * 16 acc_g) >> 4 exactly.  Within each
// 8-weight block the unpacked bytes are the even k then the odd k; the
// prologue writes x8 in the same order.
//
// Warp roles (512 threads, one CTA per SM): warp 0 streams the stages (the
// weight box and the prepared x8 tiles), warp 1 allocates TMEM and issues
// the MMAs (one thread), warps 2-7 unpack pairs of groups, warps 8-15 read
// the accumulators back (TMEM lane quarter = warp % 4, column half =
// (warp-8)/4) and fold m_g * acc_g into int64 registers.  Each role only
// waits on the one before it, through rings deep enough (4 A tiles, 8 TMEM
// accumulators) that no role stalls on a later one in steady state.  Every hand-off is
// an mbarrier; every wait is bounded and an expired wait sets DERR_TIMEOUT
// and unwinds the CTA (no copy or MMA left in flight).
//
// Work: units = (128-row tile, K split); split s covers groups
// [s*NG/S, (s+1)*NG/S) and writes its partial p to p[s][b][row]; k_bepi
// sums the S partials (integer addition: exact in any order) and runs the
// per-sequence epilogue of the op.  The LM head (S = 1) reduces its
// argmax inside the GEMM, per CTA in shared memory, then one atomicMax per
// sequence.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "f5_batch.cuh"
#include "f5_block.cuh"
#include "f5_gemv_core.cuh"
#include "f5_tc.cuh"

namespace f5 {

constexpr int BG_WORKERS = 6;      // unpack warps 2-7; warps 8-15 fold the accumulators
constexpr int BG_THREADS = 32 * (2 + BG_WORKERS + 8);
constexpr int BG_NA = 4;           // unpacked A-tile slots (16 KB each), two per group pair
constexpr int BG_NT = 8;           // TMEM accumulator buffers
constexpr int BG_WBYTES = BG_TILE * 64 * BG_GPS;   // packed weights per stage (32 KB)
constexpr int BG_SMEM_MAX = 232448 - 4096;
constexpr unsigned long long BG_WAIT_NS = 2000000000ull;

F5_DEV int bg_seg_of_tile(const BgemmArgs &a, int tile) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < BG_MAX_SEG; ++i)
    if (i < a.nseg && tile >= a.seg[i].tile_begin) s = i;
  return s;
}

template <int BPH>
__global__ void __launch_bounds__(BG_THREADS, 1) k_bgemm(const __grid_constant__ BgemmArgs a) {
  constexpr int BP = 2 * BPH;
  constexpr int XBYTES = BP * 128 * BG_GPS;
  constexpr int STAGE = BG_WBYTES + XBYTES;
  constexpr uint32_t TCOLS = BG_NT * BP < 32 ? 32 : BG_NT * BP;
  extern __shared__ uint8_t bg_dyn[];
  __shared__ __align__(8) uint64_t full[4], empty[4], afull[BG_NA], aempty[BG_NA], tfull[BG_NT], tempty[BG_NT];
  __shared__ __align__(8) uint64_t drain;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  __shared__ unsigned long long s_key[BP];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = a.ns;
  uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(bg_dyn) + 1023) & ~(uintptr_t)1023);
  uint8_t *aslot = base;                                   // BG_NA x 16 KB
  uint8_t *stg = base + BG_NA * 16384;                     // NS x STAGE
  const int gpu = a.NG / a.S;                              // groups per unit
  const int spu = gpu / BG_GPS;                            // stages per unit
  const int ppu = gpu / 2;                                 // group pairs per unit
  const int units = a.ntiles * a.S;
  const bool tr = a.trace && blockIdx.x == 0;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], BG_WORKERS + 1);   // every worker warp + the MMA commit
    }
    for (int i = 0; i < BG_NA; ++i) {
      mbar_init(&afull[i], BG_WORKERS);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < BG_NT; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);
    }
    mbar_init(&drain, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid < BP) s_key[tid] = 0ull;
  if (warp == 1) tc_alloc(&s_tmem, TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ---------------- producer ----------------
    // A stage reads 256 bytes from each of 128 rows 2112 (6336) bytes apart,
    // a poor DRAM access pattern; so each unit's rows are first streamed into
    // L2 contiguously (one bulk prefetch per row, one unit ahead) and the
    // stage boxes then hit L2.
    auto prefetch_unit = [&](int u) {
      if (u >= units) return;
      const int tile = u / a.S, sp = u % a.S;
      const BgemmSeg &sg = a.seg[bg_seg_of_tile(a, tile)];
      const int r0 = (tile - sg.tile_begin) * BG_TILE;
      const int nr = min(BG_TILE, sg.rows - r0);
      const uint8_t *b0 = sg.w + (size_t)r0 * a.stride + (size_t)sp * gpu * 64;
      for (int r = lane; r < nr; r += 32) prefetch_l2(b0 + (size_t)r * a.stride, (uint32_t)gpu * 64);
    };
    prefetch_unit(blockIdx.x);
    int sc = 0;
    for (int u = blockIdx.x; u < units && !s_abort; u += gridDim.x) {
      const int tile = u / a.S, sp = u % a.S;
      const int si = bg_seg_of_tile(a, tile);
      const int r0 = (tile - a.seg[si].tile_begin) * BG_TILE;
      prefetch_unit(u + gridDim.x);
      for (int st = 0; st < spu; ++st, ++sc) {
        const int s = sc % NS;
        bool ok = true;
        if (lane == 0 && sc >= NS) ok = mbar_wait(&empty[s], ((sc / NS) - 1) & 1, BG_WAIT_NS);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok || s_abort) {
          if (lane == 0 && !ok) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
          break;
        }
        const int g = sp * gpu + st * BG_GPS;
        uint8_t *dst = stg + (size_t)s * STAGE;
        if (tr && lane == 0 && sc < 1024) a.trace[sc] = gtimer();
        if (lane == 0) {
          // one box of 128 rows x 256 bytes (rows past the image read as zeros)
          mbar_expect_tx(&full[s], (uint32_t)STAGE);
          tma_load_2d(dst, &a.tmap[si], g * 64, r0, &full[s]);
          bulk_g2s(dst + BG_WBYTES, a.xt + (size_t)g * BP * 128, XBYTES, &full[s]);
        }
        __syncwarp();
      }
    }
    // drain: wait until every issued stage has landed (bounded)
    if (lane == 0 && s_abort)
      for (int i = max(0, sc - NS); i < sc; ++i) mbar_wait(&full[i % NS], (i / NS) & 1, BG_WAIT_NS);
  } else if (warp == 1) {
    // ---------------- MMA issuer (one thread) ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_s8s8(BG_TILE, BP);
      int sc = 0, ac = 0, tc = 0;
      bool issued = false;
      for (int u = blockIdx.x; u < units && !s_abort; u += gridDim.x) {
        for (int st = 0; st < spu && !s_abort; ++st, ++sc) {
          const int s = sc % NS;
          if (!mbar_wait(&full[s], (sc / NS) & 1, BG_WAIT_NS)) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); break; }
          const uint32_t xbase = smem_u32(stg + (size_t)s * STAGE + BG_WBYTES);
          for (int gi = 0; gi < BG_GPS; ++gi, ++ac, ++tc) {
            const int as = ac % BG_NA, ts = tc % BG_NT;
            if (!mbar_wait(&afull[as], (ac / BG_NA) & 1, BG_WAIT_NS) ||
                (tc >= BG_NT && !mbar_wait(&tempty[ts], ((tc / BG_NT) - 1) & 1, BG_WAIT_NS))) {
              s_abort = 1;
              atomicOr(a.err, DERR_TIMEOUT);
              break;
            }
            tc_fence_after();
            const uint64_t ad = sw128_desc(smem_u32(aslot + (size_t)as * 16384));
            const uint64_t bd = sw128_desc(xbase + (uint32_t)(gi * BP * 128));
#pragma unroll
            for (int k = 0; k < 4; ++k) tc_mma_i8(tmem + (uint32_t)(ts * BP), ad + 2 * k, bd + 2 * k, idesc, k > 0);
            issued = true;
            if (tr && tc < 2048) a.trace[4096 + tc] = gtimer();
            tc_commit(&aempty[as]);
            tc_commit(&tfull[ts]);
          }
          tc_commit(&empty[s]);
        }
      }
      // every MMA complete before TMEM is released
      if (issued) {
        tc_commit(&drain);
        mbar_wait(&drain, 0, BG_WAIT_NS);
      }
    }
    __syncwarp();
  } else if (warp < 2 + BG_WORKERS) {
    // ---------------- unpack (warps 2-7) ----------------
    // 8 lanes take one row's 128 contiguous packed bytes (conflict-free
    // reads) of a pair of groups; lane chunk j = 4 h + c is packed chunk c
    // of group gs + h.  Lanes of the second group store their two output
    // chunks in the opposite order, so each store phase covers 8 distinct
    // 16-byte bank groups.  Nibbles become 16 w as int8: (w << 4) & 0xF0 for
    // even k, w & 0xF0 for odd k.  Row quads (4 rows per warp instruction)
    // are dealt round-robin: warp u takes quads u, u + 6, ...
    const int wu = warp - 2;
    const int j = lane & 7, h = j >> 2, c = j & 3;
    bool ok = true;
    int sc = 0, pc = 0;
    for (int u = blockIdx.x; u < units && ok && !s_abort; u += gridDim.x) {
      for (int pi = 0; pi < ppu; ++pi, ++pc) {
        const int s = sc % NS, gs = (2 * pi) % BG_GPS;   // stage, first group within it
        if (gs == 0) {
          if (lane == 0) ok = mbar_wait(&full[s], (sc / NS) & 1, BG_WAIT_NS);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (tr && tid == 64 && sc < 1024) a.trace[1024 + sc] = gtimer();
        }
        const int ac = 2 * pc, as0 = ac % BG_NA, as1 = (ac + 1) % BG_NA;
        if (ok && ac >= BG_NA) {
          if (lane == 0)
            ok = mbar_wait(&aempty[as0], ((ac / BG_NA) - 1) & 1, BG_WAIT_NS) &&
                 mbar_wait(&aempty[as1], (((ac + 1) / BG_NA) - 1) & 1, BG_WAIT_NS);
          ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        if (!ok || s_abort) {
          if (lane == 0 && !ok) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
          ok = false;
          break;
        }
        const uint8_t *src = stg + (size_t)s * STAGE + gs * 64 + j * 16;
        uint8_t *dst = aslot + (size_t)(h ? as1 : as0) * 16384;
#pragma unroll 2
        for (int qd = wu; qd < BG_TILE / 4; qd += BG_WORKERS) {
          const int r = qd * 4 + (lane >> 3);
          const uint4 w = *reinterpret_cast<const uint4 *>(src + r * 256);
          const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
          uint32_t o[8];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            o[2 * k] = (wv[k] << 4) & 0xF0F0F0F0u;
            o[2 * k + 1] = wv[k] & 0xF0F0F0F0u;
          }
          const uint32_t o0 = sw128_off(r, c * 32), o1 = sw128_off(r, c * 32 + 16);
          const uint4 v0 = make_uint4(o[0], o[1], o[2], o[3]), v1 = make_uint4(o[4], o[5], o[6], o[7]);
          *reinterpret_cast<uint4 *>(dst + (h ? o1 : o0)) = h ? v1 : v0;
          *reinterpret_cast<uint4 *>(dst + (h ? o0 : o1)) = h ? v0 : v1;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> MMA reads
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&afull[as0]);
          mbar_arrive(&afull[as1]);
          if (gs + 2 == BG_GPS) mbar_arrive(&empty[s]);   // the stage's packed bytes are consumed
        }
        if (tr && tid == 64 && ac < 2048) a.trace[2048 + ac] = gtimer();
        if (gs + 2 == BG_GPS) ++sc;
      }
    }
  } else {
    // ---------------- accumulator fold (warps 8-15) ----------------
    const int q = warp & 3, hf = (warp - 2 - BG_WORKERS) >> 2;
    const int rt = 32 * q + lane;                              // row within the tile
    const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(hf * BPH);
    constexpr int LDW = BPH < 16 ? BPH : 16;                   // columns per TMEM load
    int tc = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok && !s_abort; u += gridDim.x) {
      const int tile = u / a.S, sp = u % a.S;
      const BgemmSeg &sg = a.seg[bg_seg_of_tile(a, tile)];
      const int r0 = (tile - sg.tile_begin) * BG_TILE;
      const bool valid = rt < sg.rows - r0;
      long long acc[BPH];
#pragma unroll
      for (int jj = 0; jj < BPH; ++jj) acc[jj] = 0;
      // group scales 8 at a time, the next 8 prefetched one block ahead
      const uint4 *ms = reinterpret_cast<const uint4 *>(sg.w + (size_t)(valid ? r0 + rt : r0) * a.stride +
                                                        (size_t)a.NG * 64 + 2 * sp * gpu);
      uint4 mv = __ldg(ms), mvn = gpu > 8 ? __ldg(ms + 1) : make_uint4(0, 0, 0, 0);
      for (int gi = 0; gi < gpu; ++gi, ++tc) {
        if ((gi & 7) == 0 && gi) {
          mv = mvn;
          if (gi + 8 < gpu) mvn = __ldg(ms + (gi >> 3) + 1);
        }
        const uint32_t mw = (gi & 6) == 0 ? mv.x : ((gi & 6) == 2 ? mv.y : ((gi & 6) == 4 ? mv.z : mv.w));
        const int32_t m = (int32_t)((gi & 1) ? (mw >> 16) : (mw & 0xFFFFu));
        const int ts = tc % BG_NT;
        if (lane == 0) ok = mbar_wait(&tfull[ts], (tc / BG_NT) & 1, BG_WAIT_NS);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok || s_abort) {
          if (lane == 0 && !ok) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
          ok = false;
          break;
        }
        if (tr && tid == 2 * 32 + BG_WORKERS * 32 && tc < 2048) a.trace[6144 + tc] = gtimer();
        tc_fence_after();
#pragma unroll
        for (int hh = 0; hh < BPH / LDW; ++hh) {
          int32_t d[LDW];
          tc_ld<LDW>(tl + (uint32_t)(ts * BP + hh * LDW), d);
          tc_wait_ld();
#pragma unroll
          for (int jj = 0; jj < LDW; ++jj) acc[hh * LDW + jj] += (long long)m * d[jj];   // 16 p
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[ts]);
        if (tr && tid == 2 * 32 + BG_WORKERS * 32 && tc < 2048) a.trace[8192 + tc] = gtimer();
      }
      if (!ok) break;
      if (sg.argmax) {
        const int row = r0 + rt;
#pragma unroll
        for (int jj = 0; jj < BPH; ++jj) {
          const int b = hf * BPH + jj;
          if (valid && b < a.B) {
            const int32_t y = finish_y32(acc[jj], a.sh, a.err, nullptr);
            atomicMax(&s_key[b], argmax_key(y, row));
          }
        }
      } else if (valid) {
        int64_t *po = a.p + ((size_t)sp * BP + hf * BPH) * a.ptot + sg.p_row0 + r0 + rt;
#pragma unroll
        for (int jj = 0; jj < BPH; ++jj)
          if (hf * BPH + jj < a.B) po[(size_t)jj * a.ptot] = acc[jj] >> 4;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tc_dealloc(tmem, TCOLS);
  if (a.key && tid < a.B && s_key[tid]) atomicMax(&a.key[tid], s_key[tid]);
}

// ---------------------------------------------------------------------------
// k_bprep: per-sequence prologue -> the GEMM's B operand
// ---------------------------------------------------------------------------
constexpr int BP_THREADS = 512;

template <int MAXB>
__global__ void __launch_bounds__(BP_THREADS) k_bprep(const __grid_constant__ BprepArgs pa) {
  extern __shared__ __align__(16) uint8_t bp_dyn[];
  __shared__ long long red[32];
  __shared__ long long s_r;
  __shared__ int s_meta[4];
  uint2 *xs = reinterpret_cast<uint2 *>(bp_dyn);
  const int b = blockIdx.y, tid = threadIdx.x;
  const int nblk = pa.K >> 3;
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (pa.pro.mode == PRO_X8) {
    const int8_t *x8 = pa.x8_in + (size_t)b * pa.K;
    for (int bb = tid; bb < nblk; bb += BP_THREADS) {
      const uint2 v = *reinterpret_cast<const uint2 *>(x8 + 8 * bb);
      xs[(((bb >> 7) << 2) + (bb & 3)) * 32 + ((bb >> 2) & 31)] =
          make_uint2(__byte_perm(v.x, v.y, 0x6420), __byte_perm(v.x, v.y, 0x7531));
    }
    if (tid == 0) {
      s_meta[0] = pa.xmeta_in ? pa.xmeta_in[2 * b] : 0;
      s_meta[1] = pa.xmeta_in ? pa.xmeta_in[2 * b + 1] : 0;
    }
  } else {
    GemvArgs ga;
    ga.K = pa.K;
    ga.err = pa.err;
    ga.abort_flag = nullptr;
    ga.pro = pa.pro;
    ga.pro.tag_op1 = 0;
    ga.pro.src = static_cast<const uint8_t *>(pa.pro.src) + b * pa.src_bs;
    if (pa.pro.src2) ga.pro.src2 = static_cast<const uint8_t *>(pa.pro.src2) + b * pa.src2_bs;
    if (pa.pro.dbg) ga.pro.dbg = pa.pro.dbg + b;
    ga.pro.xq_out.x8 = pa.x8 ? pa.x8 + (size_t)b * pa.K : nullptr;   // stored by blockIdx.x == 0
    ga.pro.xq_out.meta = pa.x8 ? pa.xmeta + 2 * b : nullptr;
    prologue<MAXB>(BlockSync(), ga, xs, red, &s_r, s_meta);
  }
  __syncthreads();
  if (tid == 0) {
    pa.xmeta[2 * b] = s_meta[0];
    pa.xmeta[2 * b + 1] = s_meta[1];
  }
  // 8-element block bb = bytes [8bb, 8bb+8) of the permuted row: group bb/16,
  // 16-byte chunk (bb%16)/2 of the group's 128-byte swizzled row b
  for (int bb = tid; bb < nblk; bb += BP_THREADS) {
    const uint2 v = xs[(((bb >> 7) << 2) + (bb & 3)) * 32 + ((bb >> 2) & 31)];
    const int g = bb >> 4;
    *reinterpret_cast<uint2 *>(pa.xt + (size_t)g * pa.Bp * 128 + sw128_off(b, (bb & 15) * 8)) = v;
  }
}

// ---------------------------------------------------------------------------
// k_bepi: per-(sequence, row) epilogue of a batched GEMM op
// ---------------------------------------------------------------------------
constexpr int BE_THREADS = 256;

__global__ void __launch_bounds__(BE_THREADS) k_bepi(const __grid_constant__ BepiArgs ea) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.y;
  const int u = blockIdx.x * BE_THREADS + threadIdx.x;
  const GemvArgs &a = ea.g;
  if (u >= a.total_units) return;
  const int si = seg_of(a, u);
  const BepiSeg &bs = ea.bs[si];
  GemvSeg sg = a.seg[si];
  const int row = u - sg.unit_begin;
  const size_t pstride = (size_t)ea.Bp * ea.ptot;
  const int64_t *pb = ea.p + (size_t)b * ea.ptot;
  long long p = 0, pu = 0;
  for (int s = 0; s < ea.S; ++s) p += pb[s * pstride + bs.p_row0 + row];
  const int e_x = ea.xmeta[2 * b], in_f = ea.xmeta[2 * b + 1];
  if (sg.out) sg.out = static_cast<uint8_t *>(sg.out) + b * bs.out_bs;
  if (sg.aux_out) sg.aux_out = static_cast<uint8_t *>(sg.aux_out) + b * bs.aux_bs;
  if (sg.p_out) sg.p_out = reinterpret_cast<int64_t *>(reinterpret_cast<uint8_t *>(sg.p_out) + b * bs.pout_bs);
  if (sg.mode == GM_SILU_MUL) {
    for (int s = 0; s < ea.S; ++s) pu += pb[s * pstride + bs.p_row0_up + row];
    epilogue_pair(a, sg, row, p << 4, pu << 4, e_x, in_f);
    return;
  }
  if (sg.mode == GM_CONV) {
    sg.aux0 = static_cast<uint8_t *>(sg.aux0) + b * bs.ring_bs;
    sg.T = &ea.params[b].T;
  }
  unsigned long long best = 0;
  epilogue_row(a, sg, row, p << 4, e_x, in_f, best);
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
bool bgemm_tmap(TmapBytes *out, const uint8_t *w, int rows, int stride) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  static_assert(sizeof(CUtensorMap) == sizeof(TmapBytes), "CUtensorMap is 128 bytes");
  const cuuint64_t dims[2] = {(cuuint64_t)stride, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)stride};
  const cuuint32_t box[2] = {256, (cuuint32_t)BG_TILE};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = encode(reinterpret_cast<CUtensorMap *>(out), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                            const_cast<uint8_t *>(w), dims, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static cudaError_t launch_ex(const void *fn, void **args, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_bprep(const BprepArgs &a, cudaStream_t st, bool pdl) {
  if (a.K % 128 || a.K > 12288 || a.B < 1 || a.B > a.Bp) return cudaErrorInvalidValue;
  const int nblk = a.K / 8;
  const size_t xs_bytes = (size_t)((nblk + 127) / 128) * 4 * 32 * sizeof(uint2);
  void *args[] = {const_cast<BprepArgs *>(&a)};
  const int maxb = (nblk + BP_THREADS - 1) / BP_THREADS;
  const void *fn = maxb <= 1 ? (const void *)k_bprep<1> : maxb <= 2 ? (const void *)k_bprep<2> : (const void *)k_bprep<3>;
  return launch_ex(fn, args, dim3(1, a.B), dim3(BP_THREADS), xs_bytes, st, pdl);
}

size_t bgemm_smem(int Bp, int *ns) {
  const size_t stage = (size_t)BG_WBYTES + (size_t)Bp * 128 * BG_GPS;
  const size_t fixed = 1024 + (size_t)BG_NA * 16384;
  int n = (int)((BG_SMEM_MAX - fixed) / stage);
  if (n > 4) n = 4;
  if (ns) *ns = n;
  return fixed + (size_t)n * stage;
}

int bgemm_splits(int tiles, int NG, int ctas, bool argmax) {
  if (argmax) return 1;
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= NG; ++s) {
    if (NG % s || (NG / s) % 8) continue;
    const long long waves = ((long long)tiles * s + ctas - 1) / ctas;
    const long long cost = waves * (NG / s) * 16 + s;   // group-steps of the busiest CTA (+ split overhead)
    if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = s; }
  }
  return best;
}

template <int BPH>
static cudaError_t launch_bg(const BgemmArgs &a, cudaStream_t st, bool pdl, int max_ctas) {
  int ns = 0;
  const size_t smem = bgemm_smem(2 * BPH, &ns);
  if (ns < 2) return cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_bgemm<BPH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  BgemmArgs b = a;
  b.ns = ns;
  const int units = a.ntiles * a.S;
  const int grid = units < max_ctas ? units : max_ctas;
  void *args[] = {&b};
  return launch_ex((const void *)k_bgemm<BPH>, args, dim3(grid), dim3(BG_THREADS), smem, st, pdl);
}

static unsigned long long *g_bg_trace = nullptr;   // process-wide trace buffer (f5_batch_trace)
unsigned long long *&bgemm_trace_buffer() { return g_bg_trace; }

cudaError_t launch_bgemm(BgemmArgs a, cudaStream_t st, bool pdl, int max_ctas) {
  if (!a.trace) a.trace = g_bg_trace;
  for (int i = 0; i < a.nseg; ++i)
    if ((reinterpret_cast<uintptr_t>(a.seg[i].w) & 15) || !bgemm_tmap(&a.tmap[i], a.seg[i].w, a.seg[i].rows, a.stride))
      return cudaErrorInvalidValue;
  if (a.K % 1024 || a.NG != a.K / 128 || a.S < 1 || a.NG % a.S || (a.NG / a.S) % 8 || a.ntiles < 1 ||
      a.B < 1 || a.B > a.Bp || a.stride % 16)
    return cudaErrorInvalidValue;
  switch (a.Bp) {
    case 16: return launch_bg<8>(a, st, pdl, max_ctas);
    case 32: return launch_bg<16>(a, st, pdl, max_ctas);
    case 64: return launch_bg<32>(a, st, pdl, max_ctas);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bepi(const BepiArgs &a, cudaStream_t st, bool pdl) {
  if (a.g.total_units < 1) return cudaSuccess;
  void *args[] = {const_cast<BepiArgs *>(&a)};
  return launch_ex((const void *)k_bepi, args, dim3((a.g.total_units + BE_THREADS - 1) / BE_THREADS, a.B),
                   dim3(BE_THREADS), 0, st, pdl);
}

}  // namespace f5
