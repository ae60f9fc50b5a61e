// Persistent decode-step kernel (sm_100a): one cooperative launch runs the
// whole batch-1 decode step of ref/fidelity_check.py:404-448 (FxRunner.step)
// over every SM, replacing the 163-launch per-op chain and its ~6-8 us of
// launch / drain / ramp cost per dependent kernel.
//
// Roles inside each CTA (one CTA per SM, 576 threads):
//  * producer (one lane of warp 16) walks the step's op list and streams
//    EVERY weight row this CTA will ever consume, in consumption order,
//    through a ring of MEGA_STAGE-byte shared-memory stages (cp.async.bulk,
//    single-destination copies, full / empty mbarriers).  Weights do not depend on
//    activations, so the stream never waits for a grid barrier: while the
//    consumers sit at a barrier or in a DeltaNet / attention core, the ring
//    fills and HBM stays busy.  It also prefetches the CTA's DeltaNet head
//    state and its attention K / V rows into a scratch region, gated by a
//    scratch-free mbarrier the consumers arrive on after each use.
//  * warp 17 has no role (an L2-prefetch warp that ran ahead of the
//    producer measured slower at every lead and was removed: the kernel is a
//    single function whose code size shows in its instruction-fetch stalls).
//  * consumers (warps 0-15, named barrier 1) run the ops in order, separated
//    by grid barriers (global counters, bounded spins): GEMV prologue /
//    row dot products / epilogues (f5_gemv_core.cuh), the DeltaNet head core
//    (f5_dn_core.cuh, dk rows split over 4 thread quarters) and a split-T
//    attention core whose three cross-CTA reductions (score max, exp sum,
//    PV sums) are exact integer atomics in L2 with two group barriers.
//
// Every wait is bounded (globaltimer); a CTA that gives up raises a global
// abort flag that every other wait polls, so the whole grid unwinds, drains
// its in-flight bulk copies and exits with DERR_TIMEOUT set.  The last CTA
// to finish decodes the argmax, advances the step parameters and re-zeroes
// the barrier counters for the next launch.
#include <climits>

#include <cuda_runtime.h>

#include "f5_luts.h"
// F5_MEGA_TRACE selects the instance this translation unit builds: 0 the
// step kernel k_mega, whose code holds no trace marks (the kernel's speed
// follows its code size), 1 the traced copy k_mega_traced that
// f5_mega_trace.cu compiles from this same source for f5_ctx_trace_step.
#ifndef F5_MEGA_TRACE
#define F5_MEGA_TRACE 0
#endif
namespace f5 {
#if F5_MEGA_TRACE
// this op's trace row (consumer thread 0 only), null when not tracing;
// declared ahead of the shared cores so their phase marks can reach it
__shared__ unsigned long long *mg_tr;
#endif
// The integer LUTs in shared memory (copied from the global tables at
// launch): every lookup of the step's prologues, epilogues and cores is a
// shared-memory read, never an L1 miss behind the weight stream.
__shared__ int32_t mg_lut_rsqrt[F5_LUT_RSQRT_N], mg_lut_recip[F5_LUT_RECIP_N], mg_lut_exp2[F5_LUT_EXP2_N],
    mg_lut_sigmoid[F5_LUT_SIGMOID_N], mg_lut_softplus[F5_LUT_SOFTPLUS_N];
}  // namespace f5
#define F5_LUT_RSQRT mg_lut_rsqrt
#define F5_LUT_RECIP mg_lut_recip
#define F5_LUT_EXP2 mg_lut_exp2
#define F5_LUT_SIGMOID mg_lut_sigmoid
#define F5_LUT_SOFTPLUS mg_lut_softplus
#if F5_MEGA_TRACE
#define F5_PRO_MARK(k)                                     \
  do {                                                     \
    if (threadIdx.x == 0 && mg_tr) mg_tr[(k)] = gtimer();  \
  } while (0)
#endif

#include "f5_dn_core.cuh"
#include "f5_gemv_core.cuh"
#include "f5_mega.cuh"

namespace f5 {

constexpr int MG_CONS = 16;
constexpr int MG_CT = MG_CONS * 32;
constexpr int MG_NS_MAX = 6;
constexpr int MG_XS = 12 * 4 * 32 * 8;          // x8 of K <= 12288 in the lane-major layout
constexpr int MG_RESB = MEGA_RES * 8;
constexpr int MG_GAINB = 4096 * 4;              // the RMSNorm gains of one K = 4096 prologue
constexpr unsigned long long MG_WAIT_NS = 1000000000ull;   // 1 s: a safety net only
using CSync = NamedSync<1, MG_CT>;

// scratch layout: DeltaNet column quarter of a head
constexpr int DN_SD = 0, DN_QN = 8192, DN_KN = DN_QN + 512, DN_PART = DN_KN + 512, DN_OG = DN_PART + 4096,
              DN_VZN = DN_OG + 1024, DN_END = DN_VZN + 3 * 32 * 8;
// scratch layout: attention (K / V fills are 16-byte aligned for cp.async.bulk)
constexpr int AT_K = 0, AT_V = AT_K + MEGA_SUB * 256, AT_KE = AT_V + MEGA_SUB * 256, AT_VE = AT_KE + MEGA_SUB,
              AT_Q16 = AT_VE + MEGA_SUB, AT_K16 = AT_Q16 + 4 * 256 * 2, AT_K8N = AT_K16 + 4 * 256 * 2,
              AT_V8N = AT_K8N + 256, AT_XN = AT_V8N + 256, AT_SC = AT_XN + 4 * 256 * 2;
static_assert(AT_SC % 16 == 0 && AT_KE % 16 == 0 && AT_VE % 16 == 0, "scratch alignment");

// ---------------------------------------------------------------------------
// bounded waits and barriers
// ---------------------------------------------------------------------------
F5_DEV unsigned ld_acquire_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
F5_DEV unsigned ld_relaxed_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct Abort {
  unsigned *flag;
  uint32_t *err;
  F5_DEV void raise() const {
    atomicOr(err, DERR_TIMEOUT);
    atomicExch(flag, 1u);
  }
  F5_DEV bool raised() const { return ld_relaxed_u32(flag) != 0; }
};

// mbarrier wait that gives up after MG_WAIT_NS or once another CTA aborted.
// The abort flag lives in L2: under a saturated weight stream one poll costs
// about a microsecond, so it is read only after MG_POLL_NS of waiting (and
// then every MG_POLL_NS), never on the normal sub-microsecond waits.
constexpr unsigned long long MG_POLL_NS = 20000ull;
F5_DEV bool mwait(uint64_t *b, uint32_t parity, const Abort &ab) {
  const uint32_t addr = smem_u32(b);
  unsigned long long t0 = 0, tpoll = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
    if (ok) return true;
    if ((it & 63) == 63) {
      const unsigned long long t = gtimer();
      if (t0 == 0) {
        t0 = t;
        tpoll = t + MG_POLL_NS;
      } else if (t >= tpoll) {
        if (ab.raised()) return false;
        if (t - t0 > MG_WAIT_NS) { ab.raise(); return false; }
        tpoll = t + MG_POLL_NS;
      }
    }
  }
}


// The producer's waits (a slot, the scratch or the gains buffer to be freed
// by the consumers): the producer lane shares a sub-partition with four
// consumer warps, so between tries it sleeps instead of spinning and takes
// no issue slots from them; a refill issued up to ~0.1 us late is hidden by
// the HBM latency it waits on anyway.
F5_DEV bool pwait(uint64_t *b, uint32_t parity, const Abort &ab) {
  const uint32_t addr = smem_u32(b);
  unsigned long long t0 = 0, tpoll = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
    if (ok) return true;
    __nanosleep(64);
    if ((it & 15) == 15) {
      const unsigned long long t = gtimer();
      if (t0 == 0) {
        t0 = t;
        tpoll = t + MG_POLL_NS;
      } else if (t >= tpoll) {
        if (ab.raised()) return false;
        if (t - t0 > MG_WAIT_NS) { ab.raise(); return false; }
        tpoll = t + MG_POLL_NS;
      }
    }
  }
}

// Counter barrier over `target` CTAs (consumer groups).  One thread's
// release add / acquire polls, bracketed by the group's named barrier, order
// every consumer thread's prior global writes before any later read in the
// other CTAs (release and acquire are cumulative over the bar.sync).
F5_DEV bool counter_barrier(const CSync &sy, unsigned *cnt, unsigned target, const Abort &ab) {
  sy.sync();
  bool bad = false;
  if (sy.tid() == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
    unsigned long long t0 = 0, tpoll = 0;
    for (uint32_t it = 0;; ++it) {
      if (ld_acquire_u32(cnt) >= target) break;
      if ((it & 7) == 7) {
        const unsigned long long t = gtimer();
        if (t0 == 0) {
          t0 = t;
          tpoll = t + MG_POLL_NS;
        } else if (t >= tpoll) {
          if (ab.raised()) { bad = true; break; }
          if (t - t0 > MG_WAIT_NS) { ab.raise(); bad = true; break; }
          tpoll = t + MG_POLL_NS;
        }
      }
    }
  }
  return !sy.any(bad);
}

// Marked 64-bit values for the attention's group exchanges: the value goes
// out as two naturally aligned 8-byte words {low or high half, marker 1} --
// each word is single-copy atomic, so a reader that sees both markers has
// the whole value, with no fence or counter.  The slots are zeroed by the
// step's BEGIN op, grid barriers before any attention op.
F5_DEV void slot_put(unsigned long long *slot, long long v) {
  const unsigned long long lo = (unsigned long long)(uint32_t)v | (1ull << 32);
  const unsigned long long hi = (unsigned long long)(uint32_t)((unsigned long long)v >> 32) | (1ull << 32);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(slot), "l"(lo) : "memory");
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(slot + 1), "l"(hi) : "memory");
}
F5_DEV bool slot_get(const unsigned long long *slot, long long &v, const Abort &ab) {
  unsigned long long t0 = 0, tpoll = 0;
  for (uint32_t it = 0;; ++it) {
    unsigned long long lo, hi;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(lo) : "l"(slot) : "memory");
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(hi) : "l"(slot + 1) : "memory");
    if ((lo >> 32) == 1ull && (hi >> 32) == 1ull) {
      v = (long long)((hi << 32) | (lo & 0xFFFFFFFFull));
      return true;
    }
    if ((it & 7) == 7) {
      const unsigned long long t = gtimer();
      if (t0 == 0) {
        t0 = t;
        tpoll = t + MG_POLL_NS;
      } else if (t >= tpoll) {
        if (ab.raised()) return false;
        if (t - t0 > MG_WAIT_NS) { ab.raise(); return false; }
        tpoll = t + MG_POLL_NS;
      }
    }
  }
}

F5_DEV void release_scratch(const CSync &sy, uint64_t *bfree) {
  sy.sync();
  if (sy.tid() == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic accesses before the next async fill
    mbar_arrive(bfree);
  }
}

// first unit of CTA b when `total` units split over G CTAs; total * G < 2^31
// here (<= 248,320 rows x the SM count), so 32-bit arithmetic is exact
F5_DEV int part_lo(int total, int G, int b) { return (int)((unsigned)total * (unsigned)b / (unsigned)G); }

// ---------------------------------------------------------------------------
// attention geometry (identical in producer and consumers)
// ---------------------------------------------------------------------------
struct AttGeo {
  bool ok;
  int pos, Tn, Told, chunk, t0, t1, kv, j, cpg;
};
F5_DEV AttGeo att_geo(const AttnArgs &a, int T, int pos, int G, int b) {
  AttGeo g;
  g.cpg = G / a.nkv;
  g.kv = b / g.cpg;
  g.j = b % g.cpg;
  g.ok = T >= 0 && T < a.max_T;
  g.pos = pos;
  if (pos < 0 || pos >= a.max_pos) { g.ok = false; g.pos = 0; }
  g.Tn = g.ok ? T + 1 : max(0, min(T, a.max_T));
  g.Told = g.ok ? T : g.Tn;
  g.chunk = (((g.Tn + g.cpg - 1) / g.cpg) + 15) & ~15;
  g.t0 = g.j * g.chunk;
  g.t1 = min(g.t0 + g.chunk, g.Tn);
  return g;
}
// cached rows of fill `s` of this CTA's token chunk: [sb, sb + n)
F5_DEV int att_fill_rows(const AttGeo &g, int s, int &sb) {
  sb = g.t0 + s * MEGA_SUB;
  const int se = min(sb + MEGA_SUB, g.t1);
  return max(0, min(se, g.Told) - sb);
}
F5_DEV void att_issue(uint8_t *dst_rows, uint8_t *dst_e, const int8_t *rows, const int8_t *ex, size_t row0, int n,
                      uint64_t *bar) {
  const uint32_t rb = (uint32_t)n * 256, eb = ((uint32_t)n + 15) & ~15u;
  mbar_expect_tx(bar, rb + eb);
  bulk_g2s(dst_rows, rows + row0 * 256, rb, bar);
  bulk_g2s(dst_e, ex + row0, eb, bar);
}

// Shared memory at namespace scope: every address below is a compile-time
// constant (no pointer kept in registers); the dynamic region's layout
// depends only on the ring depth ns (a launch parameter):
//   [ns x MEGA_STAGE ring][MG_XS x8 layout][MG_RESB row results][MG_GAINB gains][scratch]
extern __shared__ __align__(128) uint8_t mg_dyn[];
__shared__ __align__(8) uint64_t mg_full[MG_NS_MAX], mg_empty[MG_NS_MAX];
__shared__ __align__(8) uint64_t mg_bsd, mg_bsk, mg_bsv, mg_bfree, mg_bpd[2];
__shared__ __align__(8) uint64_t mg_gfull, mg_gfree;   // the gains buffer: filled by the producer, freed by the prologue
__shared__ __align__(16) MegaOp mg_cop[2], mg_pop[2];   // op i's descriptor in [i & 1]
__shared__ long long mg_red[64];
__shared__ long long mg_r, mg_gate[4], mg_att[8];
__shared__ long long mg_gat[64];   // group_gather's per-warp partials (apart from mg_red: no reuse race)
__shared__ int mg_meta[4], mg_e[2];
__shared__ int mg_cnt[7];   // issued fills: [0] ring, [1] sd, [2] sk, [3] sv (producer), [4] sk, [5] sv (consumers), [6] gains
__shared__ volatile int mg_abort;
__shared__ int mg_last;
constexpr int MG_XRES = 64;
__shared__ int16_t mg_xres[MG_XRES];      // this CTA's rows of the residual (4096-row partition)

// trace marker k (2..7) of the current op: consumer thread 0 only
#if F5_MEGA_TRACE
#define MG_MARK(k)                                                   \
  do {                                                               \
    if (threadIdx.x == 0 && mg_tr) mg_tr[(k)] = gtimer();            \
  } while (0)
#else
#define MG_MARK(k) \
  do {             \
  } while (0)
#endif

struct MegaSmem {
  int ns;
  F5_DEV uint8_t *ring() const { return mg_dyn; }
  F5_DEV uint2 *xs() const { return reinterpret_cast<uint2 *>(mg_dyn + ns * MEGA_STAGE); }
  F5_DEV long long *res() const { return reinterpret_cast<long long *>(mg_dyn + ns * MEGA_STAGE + MG_XS); }
  F5_DEV int32_t *gains() const { return reinterpret_cast<int32_t *>(mg_dyn + ns * MEGA_STAGE + MG_XS + MG_RESB); }
  F5_DEV uint8_t *scr() const { return mg_dyn + ns * MEGA_STAGE + MG_XS + MG_RESB + MG_GAINB; }
};

// position in the stage ring: stage s, lap parity ph (flips each wrap)
struct RingPos {
  int s = 0;
  uint32_t ph = 0;
  int lap = 0;   // completed wraps (saturating at 2: only "first lap or not" matters)
  F5_DEV void next(int ns) {
    if (++s == ns) {
      s = 0;
      ph ^= 1u;
      lap = lap < 2 ? lap + 1 : 2;
    }
  }
};

// ---------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------
F5_DEV void issue_desc(const MegaArgs &ma, const MegaSmem &S, int oi) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // buffer's previous generic reads
  mbar_expect_tx(&mg_bpd[oi & 1], sizeof(MegaOp));
  bulk_g2s(&mg_pop[oi & 1], ma.ops + oi, sizeof(MegaOp), &mg_bpd[oi & 1]);
}

F5_DEV void producer(const MegaArgs &ma, const MegaSmem &S, int T, int pos, const Abort &ab) {
  const int G = gridDim.x, b = blockIdx.x, ns = S.ns;
  int issued = 0, n_scr = 0, n_gain = 0;
  RingPos rp;
  bool bad = false;
  int desc_pending = -1;   // descriptor copy in flight (drained before exit)
  issue_desc(ma, S, 0);
  desc_pending = 0;
  for (int oi = 0; oi < ma.nops && !bad; ++oi) {
    if (!pwait(&mg_bpd[oi & 1], (oi >> 1) & 1, ab)) { bad = true; break; }
    desc_pending = -1;
    if (oi + 1 < ma.nops) {
      issue_desc(ma, S, oi + 1);
      desc_pending = oi + 1;
    }
    const MegaOp &op = mg_pop[oi & 1];
    const int kind = op.kind;
    if (kind == MK_GEMV) {
      const GemvArgs &a = op.g;
      if (a.pro.mode == PRO_RMSNORM) {   // the prologue's gains, ahead of the op's rows
        if (n_gain > 0 && !pwait(&mg_gfree, (n_gain - 1) & 1, ab)) { bad = true; break; }
        mbar_expect_tx(&mg_gfull, MG_GAINB);
        bulk_g2s(S.gains(), a.pro.w, MG_GAINB, &mg_gfull);
        mg_cnt[6] = ++n_gain;
      }
      int u = part_lo(a.total_units, G, b);
      const int u1 = part_lo(a.total_units, G, b + 1);
      Chunk ch;
      while (next_chunk(a, u, u1, ch)) {
        const int s = rp.s;
        if (rp.lap > 0 && !pwait(&mg_empty[s], rp.ph ^ 1u, ab)) { bad = true; break; }
        const GemvSeg &sg = a.seg[ch.seg];
        const uint32_t nb = (uint32_t)ch.n * a.stride;
        const bool pair = sg.mode == GM_SILU_MUL;
        uint8_t *dst = S.ring() + (size_t)s * MEGA_STAGE;
        mbar_expect_tx(&mg_full[s], pair ? 2 * nb : nb);
        bulk_g2s_stream(dst, sg.w + (size_t)ch.r0 * a.stride, nb, &mg_full[s]);
        if (pair) bulk_g2s_stream(dst + nb, sg.w2 + (size_t)ch.r0 * a.stride, nb, &mg_full[s]);
        mg_cnt[0] = ++issued;
        rp.next(ns);
      }
    } else if (kind == MK_DN) {
      if (b < 4 * ma.dn_heads) {   // head b / 4, column quarter b % 4: one contiguous 8 KB block
        if (n_scr > 0 && !pwait((&mg_bfree), (n_scr - 1) & 1, ab)) { bad = true; break; }
        mbar_expect_tx((&mg_bsd), 8192);
        bulk_g2s(S.scr() + DN_SD, op.d.S + (size_t)(b >> 2) * 16384 + (size_t)(b & 3) * 4096, 8192, (&mg_bsd));
        mg_cnt[1] += 1;
        ++n_scr;
      }
    } else if (kind == MK_ATTN) {
      const AttnArgs &a = op.at.a;
      const AttGeo g = att_geo(a, T, pos, G, b);
      if (g.kv < a.nkv) {
        if (n_scr > 0 && !pwait((&mg_bfree), (n_scr - 1) & 1, ab)) { bad = true; break; }
        int sb;
        const int n = att_fill_rows(g, 0, sb);
        if (n > 0) {
          const size_t row0 = (size_t)g.kv * a.max_T + sb;
          att_issue(S.scr() + AT_K, S.scr() + AT_KE, a.k8, a.ke, row0, n, (&mg_bsk));
          att_issue(S.scr() + AT_V, S.scr() + AT_VE, a.v8, a.ve, row0, n, (&mg_bsv));
          mg_cnt[2] += 1;
          mg_cnt[3] += 1;
        }
        ++n_scr;
      }
    }
  }
  if (desc_pending >= 0) mbar_wait(&mg_bpd[desc_pending & 1], (desc_pending >> 1) & 1, MG_WAIT_NS);
}

// ---------------------------------------------------------------------------
// consumers: GEMV
// ---------------------------------------------------------------------------
// Epilogue operands that do not depend on this step (conv ring and weights,
// the decay gate's constants) are pulled into L1 by the row's epilogue
// thread right after the prologue, so the epilogue's cached loads of them
// hit L1 (no acquire invalidates L1 inside an op).
F5_DEV void epi_prefetch(const GemvArgs &a, int uu) {
  const GemvSeg &sg = a.seg[seg_of(a, uu)];
  const int orow = sg.out_row0 + (uu - sg.unit_begin);
  const void *p0 = nullptr, *p1 = nullptr;
  if (sg.mode == GM_CONV) {
    p0 = static_cast<const int16_t *>(sg.aux0) + (size_t)orow * 4;
    p1 = static_cast<const int32_t *>(sg.aux1) + (size_t)orow * 4;
  } else if (sg.mode == GM_GATE_A) {
    p0 = static_cast<const int32_t *>(sg.aux0) + orow;
    p1 = static_cast<const int32_t *>(sg.aux1) + orow;
  }
  if (p0) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p0));
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p1));
  }
}
// The persistent kernel's row epilogue: the residual rows come from and go
// back to mg_xres (the CTA wrote them last: BEGIN and every residual op use
// the same 4096-row partition); everything else is the shared epilogue_row.
F5_DEV void mega_epilogue_row(const GemvArgs &a, const GemvSeg &sg, int i, int uu, long long acc, int e_x, int in_f,
                              uint32_t epoch, RStat &rs, int T) {
  const int row = uu - sg.unit_begin, orow = sg.out_row0 + row;
  const uint32_t tag = (epoch && sg.tag_op1) ? mk_tag(epoch, sg.tag_op1) : 0u;
  if (!(sg.mode == GM_RESID && tag && i < MG_XRES)) {
    unsigned long long unused = 0ull;
    epilogue_row<true>(a, sg, row, acc, e_x, in_f, unused, epoch, sg.rstat ? &rs : nullptr, T);
    return;
  }
  const int32_t y = finish_y32(acc, a.sh, a.err, nullptr);
  const long long v = clip16(shift_to(y, (15 - sg.e - a.sh) - e_x + in_f - sg.out_f));
  const int32_t nv = clip16((int64_t)mg_xres[i] + v);
  mg_xres[i] = (int16_t)nv;
  if (sg.rstat) rs.add(nv);
  st_tagged(a, static_cast<uint32_t *>(sg.out) + orow, tag_word(tag, nv));
}
// The split-K GEMV's epilogue: the step program emits it only for the MLP
// down projection, a tagged residual add whose rows (<= 4096 / 128 per CTA)
// all sit in mg_xres; anything else raises DERR_RANGE.  Only this law is
// compiled into the split loop: the kernel is one function whose speed
// follows its code size.
F5_DEV void mega_epilogue_resid(const GemvArgs &a, const GemvSeg &sg, int i, int uu, long long acc, int e_x,
                                int in_f, uint32_t epoch, RStat &rs) {
  const int orow = sg.out_row0 + (uu - sg.unit_begin);
  const uint32_t tag = (epoch && sg.tag_op1) ? mk_tag(epoch, sg.tag_op1) : 0u;
  if (!(sg.mode == GM_RESID && tag && i < MG_XRES)) {
    atomicOr(a.err, DERR_RANGE);
    return;
  }
  const int32_t y = finish_y32(acc, a.sh, a.err, nullptr);
  const long long v = clip16(shift_to(y, (15 - sg.e - a.sh) - e_x + in_f - sg.out_f));
  const int32_t nv = clip16((int64_t)mg_xres[i] + v);
  mg_xres[i] = (int16_t)nv;
  if (sg.rstat) rs.add(nv);
  st_tagged(a, static_cast<uint32_t *>(sg.out) + orow, tag_word(tag, nv));
}
// K = 4096 (every GEMV of the step but the MLP down projection): one row per
// consumer warp per 16-row stage.  The consumer loop is issue-bound, so it is
// kept to the row's own arithmetic: chunks are walked segment by segment
// (the same split as next_chunk, which the producer uses), K and the group
// size are compile-time constants (the host admits only g = 128), the row
// sum uses two redux.sync adds, and the LM head's argmax epilogue is batched
// -- lane k % 32 of a warp holds the warp's k-th row sum, and every 32 rows
// all lanes turn their rows into (y32, row) keys at once.
F5_DEV bool c_gemv4096(const GemvArgs &a, const MegaSmem &S, RingPos &rp, const Abort &ab, uint32_t epoch,
                       int &w_g, int T) {
  const CSync sy;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x, ns = S.ns;
  // the op's row partition and epilogue operands first: none depends on the
  // input vector, so this runs while the prologue's inputs are still in flight
  const int u0 = part_lo(a.total_units, G, b), u1 = part_lo(a.total_units, G, b + 1);
  const int stride = a.stride, sh = a.sh;
  const bool argmax = a.seg[0].mode == GM_ARGMAX;
  if (!argmax && tid < u1 - u0) epi_prefetch(a, u0 + tid);
  // RMSNorm gains: the producer's copy in shared memory (in place long before)
  const bool rms = a.pro.mode == PRO_RMSNORM;
  bool got = true;
  if (rms) {
    got = mwait(&mg_gfull, w_g & 1, ab);
    ++w_g;
  }
  prologue<1>(sy, a, S.xs(), mg_red, (&mg_r), mg_meta, epoch, rms ? S.gains() : nullptr);
  if (sy.any(!got)) return false;
  if (rms && tid == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the gains reads before the next fill
    mbar_arrive(&mg_gfree);
  }
  MG_MARK(2);
  const int e_x = mg_meta[0], in_f = mg_meta[1];
  uint2 xr[4][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) xr[c][j] = S.xs()[((c << 2) + j) * 32 + lane];
  long long *res = S.res();
  int32_t *logits = static_cast<int32_t *>(a.seg[0].out);   // argmax: optional y32 of every row
  unsigned long long best = 0ull;
  long long hold = 0;
  int hold_row = -1, k = 0;
  auto flush = [&]() {
    if (hold_row >= 0) {
      const long long y = rshr(hold >> 4, sh);
      if (y >= (1ll << 31) || y <= -(1ll << 31)) atomicOr(a.err, DERR_Y32_OVERFLOW);
      const unsigned long long key = argmax_key((int32_t)y, hold_row);
      best = key > best ? key : best;
      if (logits) logits[hold_row] = (int32_t)y;
    }
    hold_row = -1;
  };
  bool bad = false;
  int u = u0;
  if (!argmax) {
    // Two groups of eight warps share the op's stages: stage s always goes
    // to group s % 2, so each group waits on its own stages' full barriers
    // lap after lap and a parity wait can never alias an earlier lap (with
    // chunk j going to group j % 2 and an odd ring depth, a stage alternated
    // between the groups and a group could pass the wait on a phase still
    // pending for the other).  A stage holds <= 16 rows (rows_per_stage <=
    // 16) and warp w of the group reduces rows w and w + 8 together, so every
    // wait, arrival and loop step is shared by two rows.  Each warp arrives
    // with count 2, keeping the empty barrier's 16 arrivals per stage.
    const int grp = warp >> 3, wl = warp & 7;
    while (u < u1 && !bad) {
      const int si = seg_of(a, u);
      const GemvSeg &sg = a.seg[si];
      const int seg_hi = min(u1, si + 1 < a.nseg ? a.seg[si + 1].unit_begin : a.total_units);
      const bool pair = sg.mode == GM_SILU_MUL;
      const int ru = pair ? (a.rows_per_stage >> 1) : a.rows_per_stage;
      while (u < seg_hi) {
        const int n = min(ru, seg_hi - u);
        if ((rp.s & 1) == grp) {
          if (mg_abort || !mwait(&mg_full[rp.s], rp.ph, ab)) {
            mg_abort = 1;
            bad = true;
            break;
          }
          const int nrows = pair ? 2 * n : n;
          const uint8_t *st = S.ring() + rp.s * MEGA_STAGE;
          const int cbase = u - u0;
          const int r1 = wl + 8;
          // result slot of stage row r: paired stages hold n gate rows, then n up rows
          const int i0 = pair ? 2 * (cbase + wl) : cbase + wl;   // wl < n whenever r1 < nrows
          if (r1 < nrows) {
            long long p0, p1;
            row_dot4096x2(st + wl * stride, st + r1 * stride, lane, xr, p0, p1);
            const long long s0 = warp_sum_row(p0), s1 = warp_sum_row(p1);
            const int i1 = pair ? (r1 < n ? 2 * (cbase + r1) : 2 * (cbase + r1 - n) + 1) : cbase + r1;
            if (lane == 0) {
              res[i0] = s0;
              res[i1] = s1;
            }
          } else if (wl < nrows) {
            const long long s0 = warp_sum_row(row_dot4096(st + wl * stride, lane, xr));
            const int ix = pair ? (wl < n ? 2 * (cbase + wl) : 2 * (cbase + wl - n) + 1) : cbase + wl;
            if (lane == 0) res[ix] = s0;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive_cnt(&mg_empty[rp.s], 2);
        }
        rp.next(ns);
        u += n;
      }
    }
    u = u1;
  }
  while (u < u1 && !bad) {
    const int si = seg_of(a, u);
    const GemvSeg &sg = a.seg[si];
    const int seg_hi = min(u1, si + 1 < a.nseg ? a.seg[si + 1].unit_begin : a.total_units);
    const bool pair = sg.mode == GM_SILU_MUL;
    const int ru = pair ? (a.rows_per_stage >> 1) : a.rows_per_stage;
    const int orow0 = sg.out_row0 - sg.unit_begin;   // output row of unit v: orow0 + v
    while (u < seg_hi) {
      const int n = min(ru, seg_hi - u);
      if (mg_abort || !mwait(&mg_full[rp.s], rp.ph, ab)) {
        mg_abort = 1;
        bad = true;
        break;
      }
      const uint8_t *st = S.ring() + rp.s * MEGA_STAGE;
      const int nrows = pair ? 2 * n : n;
      const int cbase = u - u0;
      for (int r = warp; r < nrows; r += MG_CONS) {
        const long long acc = warp_sum_row(row_dot4096(st + r * stride, lane, xr));
        if (argmax) {
          if (lane == (k & 31)) {
            hold = acc;
            hold_row = orow0 + u + r;
          }
          if ((++k & 31) == 0) flush();
        } else if (lane == 0) {
          res[pair ? (r < n ? 2 * (cbase + r) : 2 * (cbase + r - n) + 1) : cbase + r] = acc;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&mg_empty[rp.s]);
      rp.next(ns);
      u += n;
    }
  }
  if (sy.any(bad)) return false;
  MG_MARK(3);
  if (argmax) {
    flush();
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if (lane == 0 && best) atomicMax(a.argmax_key, best);
    return true;
  }
  RStat rs;
  for (int i = tid; i < u1 - u0; i += MG_CT) {
    const int uu = u0 + i;
    const GemvSeg &sg = a.seg[seg_of(a, uu)];
    if (sg.mode == GM_SILU_MUL) epilogue_pair(a, sg, uu - sg.unit_begin, res[2 * i], res[2 * i + 1], e_x, in_f, epoch);
    else mega_epilogue_row(a, sg, i, uu, res[i], e_x, in_f, epoch, rs, T);
  }
  if (a.nseg == 1 && a.seg[0].rstat) rstat_flush(a.seg[0].rstat, rs);
  return true;
}

// K = NP * 4096 (the MLP down projection, NP = 3): a stage holds only
// MEGA_STAGE / stride rows, so each row is split into NP K-parts of 4096 and
// warp w reduces part w % NP of row w / NP against its x8 slice held in
// registers.  The partial sums are exact integers; the deferred epilogue adds
// the NP partials of a row (order-free) before the group-scale law's shift.
template <int NP>
F5_DEV bool c_gemv_split(const GemvArgs &a, const MegaSmem &S, RingPos &rp, const Abort &ab, uint32_t epoch) {
  const CSync sy;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x, ns = S.ns;
  const int K2 = a.K >> 1;
  const int u0 = part_lo(a.total_units, G, b), u1 = part_lo(a.total_units, G, b + 1);
  prologue<(NP * 4 * 128 + MG_CT - 1) / MG_CT>(sy, a, S.xs(), mg_red, (&mg_r), mg_meta, epoch);
  sy.sync();
  MG_MARK(2);
  const int e_x = mg_meta[0], in_f = mg_meta[1];
  const int part = warp % NP, wrow = warp / NP;   // warps >= NP * (16 / NP) idle
  uint2 xr[4][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) xr[c][j] = S.xs()[(((part * 4 + c) << 2) + j) * 32 + lane];
  bool bad = false;
  int u = u0;
  Chunk ch;
  while (next_chunk(a, u, u1, ch)) {
    const int s = rp.s;
    if (mg_abort || !mwait(&mg_full[s], rp.ph, ab)) {
      mg_abort = 1;
      bad = true;
      break;
    }
    if (wrow < ch.n && warp < NP * (MG_CONS / NP)) {
      const uint8_t *row = S.ring() + (size_t)s * MEGA_STAGE + (size_t)wrow * a.stride;
      long long acc = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int boff = (part * 4 + c) * 512 + lane * 16;
        const uint4 w = *reinterpret_cast<const uint4 *>(row + boff);
        const uint32_t m = *reinterpret_cast<const uint16_t *>(row + K2 + 2 * (boff >> 6));
        acc += (long long)m * dot32(w, xr[c][0], xr[c][1], xr[c][2], xr[c][3]);
      }
      acc = warp_sum_row(acc);
      if (lane == 0) S.res()[NP * (ch.u - u0 + wrow) + part] = acc;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&mg_empty[s]);
    rp.next(ns);
  }
  if (sy.any(bad)) return false;
  MG_MARK(3);
  RStat rs;
  for (int i = tid; i < u1 - u0; i += MG_CT) {
    const int uu = u0 + i;
    const GemvSeg &sg = a.seg[seg_of(a, uu)];
    long long acc = 0;
#pragma unroll
    for (int p = 0; p < NP; ++p) acc += S.res()[NP * i + p];
    if (i == 0) MG_MARK(4);
    mega_epilogue_resid(a, sg, i, uu, acc, e_x, in_f, epoch, rs);
    if (i == 0) MG_MARK(5);
  }
  if (a.nseg == 1 && a.seg[0].rstat) rstat_flush(a.seg[0].rstat, rs);
  return true;
}

// ---------------------------------------------------------------------------
// consumers: DeltaNet (ref/layer_fixed.py:1522-1580), one column quarter of a
// head per CTA (CTAs [0, 4 * heads)).  The recurrence of a state column is
// independent of the other columns (kv_mem, delta, the rank-1 update and o
// are all per column), so the quarter runs locally on its 128 x 32 slice;
// only the head-wide block-float shift and gated norm need all 128 o values,
// which the four CTAs of a head exchange through marked slots.  Thread
// (warp w, lane l) owns column 32 q + l, rows 8 w .. 8 w + 7.
// ---------------------------------------------------------------------------
// plain or dataflow-tagged scalar input (tagged: polled until ready)
F5_DEV long long ld_in16(const int16_t *p, int i, uint32_t tag, const Abort &ab) {
  if (!tag) return __ldcg(p + i);
  uint32_t w[1];
  ld_tagged<1>(reinterpret_cast<const uint32_t *>(p) + i, tag, w, ab.flag, ab.err);
  return tag_s16(w[0]);
}
F5_DEV long long ld_inu(const int32_t *p, int i, uint32_t tag, const Abort &ab) {   // unsigned 16-bit gates
  if (!tag) return __ldcg(p + i);
  uint32_t w[1];
  ld_tagged<1>(reinterpret_cast<const uint32_t *>(p) + i, tag, w, ab.flag, ab.err);
  return (long long)(w[0] & 0xFFFFu);
}

F5_DEV bool c_dn(const MegaArgs &ma, const DnArgs &d, const MegaSmem &S, int &w_sd, const Abort &ab,
                 uint32_t epoch) {
  const int b = blockIdx.x;
  if (b >= 4 * ma.dn_heads) return true;
  const CSync sy;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = b >> 2, qd = b & 3, kh = h / d.vrep;
  uint8_t *scr = S.scr();
  int16_t *sd = reinterpret_cast<int16_t *>(scr + DN_SD);   // [128 dk][32]
  int32_t *qn = reinterpret_cast<int32_t *>(scr + DN_QN), *kn = reinterpret_cast<int32_t *>(scr + DN_KN);
  long long *part = reinterpret_cast<long long *>(scr + DN_PART);   // [16 warps][32]
  long long *vzn = reinterpret_cast<long long *>(scr + DN_VZN);     // v, z, norm_w of the quarter

  // ---- every input in one round of loads (tagged: each polled until ready) ----
  const uint32_t itag = (epoch && d.in_tag_op1) ? mk_tag(epoch, d.in_tag_op1) : 0u;
  long long qv = 0, kv = 0;
  const long long nw_pre = (tid >= 128 && tid < 160) ? __ldcg(d.norm_w + qd * 32 + tid - 128) : 0;
  if (itag && tid <= 160) {   // each thread's two tagged words polled together
    const uint32_t *c32 = reinterpret_cast<const uint32_t *>(d.qkvc);
    const int i = tid - 128, dv = qd * 32 + i;
    const uint32_t *const pw[2] = {
        tid < 128 ? c32 + kh * 128 + tid
                  : (tid < 160 ? c32 + 2 * d.lkd + h * 128 + dv : reinterpret_cast<const uint32_t *>(d.beta) + h),
        tid < 128 ? c32 + d.lkd + kh * 128 + tid
                  : (tid < 160 ? reinterpret_cast<const uint32_t *>(d.z16) + h * 128 + dv
                               : reinterpret_cast<const uint32_t *>(d.decay) + h)};
    const bool act[2] = {true, true};
    uint32_t w2[2];
    ld_tagged_multi<2>(pw, act, itag, w2, ab.flag, ab.err);
    if (tid < 128) {
      qv = tag_s16(w2[0]);
      kv = tag_s16(w2[1]);
    } else if (tid < 160) {
      vzn[i] = tag_s16(w2[0]);
      vzn[32 + i] = tag_s16(w2[1]);
      vzn[64 + i] = nw_pre;
    } else {
      mg_gate[0] = (long long)(w2[0] & 0xFFFFu);
      mg_gate[1] = (long long)(w2[1] & 0xFFFFu);
    }
  } else if (tid < 128) {
    qv = ld_in16(d.qkvc, kh * 128 + tid, itag, ab);
    kv = ld_in16(d.qkvc, d.lkd + kh * 128 + tid, itag, ab);
  } else if (tid < 160) {
    const int i = tid - 128, dv = qd * 32 + i;
    vzn[i] = ld_in16(d.qkvc, 2 * d.lkd + h * 128 + dv, itag, ab);
    vzn[32 + i] = ld_in16(d.z16, h * 128 + dv, itag, ab);
    vzn[64 + i] = __ldcg(d.norm_w + dv);
  } else if (tid == 160) {
    mg_gate[0] = ld_inu(d.beta, h, itag, ab);
    mg_gate[1] = ld_inu(d.decay, h, itag, ab);
  }
  // ---- l2norm of q and k (ref/layer_fixed.py:1322-1330): both sums in one
  // round; the q / k rsqrt by the threads that use them (uniform inputs) ----
  long long ssq, ssk;
  g_sum2_split(sy, qv * qv, kv * kv, mg_red, ssq, ssk);
  if (tid < 128) {
    int64_t rq, rk;
    int eq, ek;
    rsqrt_q((uint64_t)(ssq == 0 ? 1 : ssq), 2 * QKV_F, rq, eq);
    rsqrt_q((uint64_t)(ssk == 0 ? 1 : ssk), 2 * QKV_F, rk, ek);
    const long long q16 = clip16(rshr(qv * rq, QKV_F + 30 - eq - NRM_F));
    qn[tid] = (int32_t)rshr(q16 * 2896, 15);    // round(2^15 / sqrt(128)) = 2896
    kn[tid] = (int32_t)clip16(rshr(kv * rk, QKV_F + 30 - ek - NRM_F));
  }
  MG_MARK(2);
  const bool got = mwait((&mg_bsd), w_sd & 1, ab);
  ++w_sd;
  if (sy.any(!got)) return false;   // also publishes qn, kn, vzn, the gates
  MG_MARK(3);

  // ---- recurrence (ref/layer_fixed.py:1545-1560) ----
  const int decay = (int)mg_gate[1];
  long long kvm = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int dk = warp * 8 + i;
    const int s0 = rshr32p((int32_t)sd[dk * 32 + lane] * decay, GAT_F);   // |S*decay| < 2^30
    sd[dk * 32 + lane] = (int16_t)s0;
    kvm += (long long)(s0 * kn[dk]);                                      // |s0 * kn| < 2^30
  }
  part[warp * 32 + lane] = kvm;
  sy.sync();
  kvm = 0;
#pragma unroll
  for (int w = 0; w < MG_CONS; ++w) kvm += part[w * 32 + lane];
  kvm = rshr(kvm, NRM_F);
  const long long delta = rshr(((vzn[lane] << (S_F - QKV_F)) - kvm) * mg_gate[0], GAT_F);
  sy.sync();   // part is reused below
  long long o = 0;
  int sat = 0;
  int16_t *Sg = d.S + (size_t)h * 16384 + (size_t)qd * 4096;
  const unsigned long long dabs = uabs(delta);
  if (dabs < (1ull << 24)) {
    // |delta| < 2^24 (always, for beta <= 2^15): the rank-1 term in 32-bit
    // integers, rshr(kn * delta, NRM_F) = sign(kn * delta) * (|kn| dh +
    // ((|kn| dl + 2^(NRM_F-1)) >> NRM_F)) with |delta| = dh 2^NRM_F + dl
    // (the same split as dn_head_rec); 8 terms of |sn * qn| <= 2^15 * 2896
    // stay inside int32
    const int32_t dh = (int32_t)(dabs >> NRM_F), dl = (int32_t)(dabs & ((1u << NRM_F) - 1));
    const int32_t sdl = delta < 0 ? -1 : 0;
    int32_t o32 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int dk = warp * 8 + i;
      const int32_t k = kn[dk], ak = k < 0 ? -k : k, sg = (k >> 31) ^ sdl;
      const int32_t r = ak * dh + ((ak * dl + (1 << (NRM_F - 1))) >> NRM_F);
      int32_t sn = (int32_t)sd[dk * 32 + lane] + ((r ^ sg) - sg);
      sat += (uint32_t)(sn + 32767) > 65534u;   // |Sh| > 32767 (ref/layer_fixed.py:1557)
      sn = min(max(sn, -32768), 32767);
      Sg[dk * 32 + lane] = (int16_t)sn;
      o32 += sn * qn[dk];
    }
    o = o32;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int dk = warp * 8 + i;
      long long sn = (long long)sd[dk * 32 + lane] + rshr((long long)kn[dk] * delta, NRM_F);
      if (sn > 32767 || sn < -32767) ++sat;   // |Sh| > 32767 (ref/layer_fixed.py:1557)
      sn = clip16(sn);
      Sg[dk * 32 + lane] = (int16_t)sn;
      o += sn * qn[dk];
    }
  }
  if (d.stats && sat) atomicAdd(d.stats, (unsigned long long)sat);
  part[warp * 32 + lane] = o;
  sy.sync();
  MG_MARK(4);

  unsigned long long *xsl = d.xslots + (size_t)h * 128 * 2;
  if (d.norm_mode == 0) {
    // ---- float gated norm: each CTA outputs its own 32 columns (warp 0, lane
    // = column), so the four quarters exchange only their max |o| and their
    // wrapping (numpy int64, order-free) sum of o*o ----
    bool ok = true;
    long long ot = 0;
    unsigned long long om = 0ull, ssu = 0ull;
    if (warp == 0) {
#pragma unroll
      for (int w = 0; w < MG_CONS; ++w) ot += part[w * 32 + lane];
      ot = rshr(ot, NRM_F);
      unsigned long long qm = uabs(ot), qs = (unsigned long long)ot * (unsigned long long)ot;
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const unsigned long long u = __shfl_xor_sync(0xffffffffu, qm, o);
        qm = u > qm ? u : qm;
        qs += __shfl_xor_sync(0xffffffffu, qs, o);
      }
      if (lane == 0) {
        slot_put(xsl + (size_t)(2 * qd) * 2, (long long)qm);
        slot_put(xsl + (size_t)(2 * qd + 1) * 2, (long long)qs);
      }
      __syncwarp();
      long long v = 0;
      if (lane < 8) ok = slot_get(xsl + (size_t)lane * 2, v, ab);   // even lanes: maxima, odd: sums
      unsigned long long mx = (lane < 8 && (lane & 1) == 0) ? (unsigned long long)v : 0ull;
      unsigned long long sm = (lane < 8 && (lane & 1)) ? (unsigned long long)v : 0ull;
#pragma unroll
      for (int o = 4; o; o >>= 1) {
        const unsigned long long u = __shfl_xor_sync(0xffffffffu, mx, o);
        mx = u > mx ? u : mx;
        sm += __shfl_xor_sync(0xffffffffu, sm, o);
      }
      om = __shfl_sync(0xffffffffu, mx, 0);
      ssu = __shfl_sync(0xffffffffu, sm, 0);
    }
    if (sy.any(!ok)) return false;
    MG_MARK(5);
    if (warp == 0) {
      // block-float k_h (ref/layer_fixed.py:470-486), norm scale (:509-546)
      const int kh_shift = bf_shift(om);
      const long long o16 = clip16(kh_shift >= 0 ? rshr(ot, kh_shift) : (long long)((unsigned long long)ot << (-kh_shift)));
      const long long m = dn_norm_scale((long long)ssu, kh_shift, 128);
      const long long tt = clip16(rshr(o16 * m, 15));
      const long long nh = clip16(rshr(tt * vzn[64 + lane], 14));
      const long long zg = clip16(silu_q(vzn[32 + lane] << (12 - QKV_F)));
      const int32_t ov16 = clip16(rshr(nh * zg, 12));
      const int col = h * 128 + qd * 32 + lane;
      if (epoch && d.out_tag_op1)
        reinterpret_cast<uint32_t *>(d.on16)[col] = tag_word(mk_tag(epoch, d.out_tag_op1), ov16);
      else
        d.on16[col] = (int16_t)ov16;
      if (qd == 0 && lane == 0 && d.kh_out) d.kh_out[h] = kh_shift;
    }
    release_scratch(sy, (&mg_bfree));
    MG_MARK(6);
    return true;
  }
  // ---- eps gated norm: its sum needs k_h first, so the head's 128 o values
  // are published by quarter and gathered by all four CTAs ----
  if (warp == 0) {
    long long ot = 0;
#pragma unroll
    for (int w = 0; w < MG_CONS; ++w) ot += part[w * 32 + lane];
    slot_put(xsl + (size_t)(qd * 32 + lane) * 2, rshr(ot, NRM_F));
  }
  long long ov = 0;
  bool ok = true;
  if (tid < 128) ok = slot_get(xsl + (size_t)tid * 2, ov, ab);
  if (sy.any(!ok)) return false;
  MG_MARK(5);
  // block-float k_h (ref/layer_fixed.py:470-486), then the EPS-NORM law
  // (ref/layer_fixed.py:694-781) over the shifted values; identical in the
  // four CTAs
  const unsigned long long om = g_max_ull(sy, tid < 128 ? uabs(ov) : 0ull, reinterpret_cast<unsigned long long *>(mg_red));
  const int kh_shift = bf_shift(om);
  const long long o16 = clip16(kh_shift >= 0 ? rshr(ov, kh_shift) : (long long)((unsigned long long)ov << (-kh_shift)));
  const long long m = eps_norm_scale(g_sum_ll(sy, o16 * o16, mg_red), kh_shift, 7);
  if (tid >= qd * 32 && tid < qd * 32 + 32) {
    const int i = tid - qd * 32;
    const long long tt = clip16(rshr(o16 * m, 15));
    const long long nh = clip16(rshr(tt * vzn[64 + i], 14));
    const long long zg = clip16(silu_q(vzn[32 + i] << (12 - QKV_F)));
    const int32_t ov16 = clip16(rshr(nh * zg, 12));
    if (epoch && d.out_tag_op1)
      reinterpret_cast<uint32_t *>(d.on16)[h * 128 + tid] = tag_word(mk_tag(epoch, d.out_tag_op1), ov16);
    else
      d.on16[h * 128 + tid] = (int16_t)ov16;
  }
  if (qd == 0 && tid == 0 && d.kh_out) d.kh_out[h] = kh_shift;
  release_scratch(sy, (&mg_bfree));
  MG_MARK(6);
  return true;
}

// ---------------------------------------------------------------------------
// consumers: attention (ref/layer_fixed.py:1383-1449)
// ---------------------------------------------------------------------------
// RMSNorm(1+w) over a 256-dim head (ref/layer_fixed.py:1242-1278) then
// rope_fx on the first `rot` dims (ref/layer_fixed.py:1340-1348), for the four
// q heads and the one k head at once: thread t owns dims e and e+128
// (e = t & 127) of q head t>>7, and threads t < 128 the same dims of k.  The
// five sums share one barrier round.  q goes to q16 (shared), k stays in the
// registers k0 / k1 of threads t < 128.
F5_DEV void norm_rope_qk(const CSync &sy, long long qx0, long long qx1, long long qw0, long long qw1, long long kx0,
                         long long kx1, long long kw0, long long kw1, long long cosv, long long sinv, int rot,
                         int16_t *qn, int16_t *kn, int16_t *q16, long long &k0, long long &k1, long long *red) {
  const int t = sy.tid(), hs = t >> 7, e = t & 127, warp = t >> 5, lane = t & 31;
  const bool kt = t < 128;
  const long long ssq = warp_sum_ll(qx0 * qx0 + qx1 * qx1);
  const long long ssk = warp_sum_ll(kx0 * kx0 + kx1 * kx1);
  if (lane == 0) {
    red[warp] = ssq;
    red[16 + warp] = ssk;
  }
  sy.sync();
  auto nrm = [&](long long tot, long long x0, long long x1, long long w0, long long w1, long long &n0, long long &n1) {
    int64_t r;
    int ee;
    rsqrt_q((uint64_t)(tot == 0 ? 1 : tot), 2 * QKV_F + 8, r, ee);   // n = 256
    n0 = clip16(rshr(clip(rshr(x0 * r, 30 - ee), -(1ll << 32), (1ll << 32) - 1) * (w0 + (1 << 14)), 14));
    n1 = clip16(rshr(clip(rshr(x1 * r, 30 - ee), -(1ll << 32), (1ll << 32) - 1) * (w1 + (1 << 14)), 14));
  };
  long long n0, n1, m0 = 0, m1 = 0;
  nrm(red[4 * hs] + red[4 * hs + 1] + red[4 * hs + 2] + red[4 * hs + 3], qx0, qx1, qw0, qw1, n0, n1);
  qn[hs * 256 + e] = (int16_t)n0;
  qn[hs * 256 + e + 128] = (int16_t)n1;
  if (kt) {
    nrm(red[16] + red[17] + red[18] + red[19], kx0, kx1, kw0, kw1, m0, m1);
    kn[e] = (int16_t)m0;
    kn[e + 128] = (int16_t)m1;
  }
  sy.sync();
  const int hh = rot >> 1;
  long long o0 = n0;
  if (e < rot) {   // rot <= 128: dims e + 128 are never rotated
    const long long rr = e < hh ? -(long long)qn[hs * 256 + e + hh] : (long long)qn[hs * 256 + e - hh];
    o0 = clip16(rshr(n0 * cosv + rr * sinv, ROPE_F));
  }
  q16[hs * 256 + e] = (int16_t)o0;
  q16[hs * 256 + e + 128] = (int16_t)n1;
  k0 = m0;
  k1 = m1;
  if (kt && e < rot) {
    const long long rr = e < hh ? -(long long)kn[e + hh] : (long long)kn[e - hh];
    k0 = clip16(rshr(m0 * cosv + rr * sinv, ROPE_F));
  }
}

// Gather the cpg CTAs' marked per-head values of one phase and combine them
// per head (max or sum) into mg_att[0..3]: thread t < 4 cpg polls entry t
// (CTA t / 4, head t % 4); lanes sharing t % 4 combine by shuffles, then
// across warps.  Also a barrier of the consumer group.
F5_DEV bool group_gather(const CSync &sy, const unsigned long long *slots, int cpg, bool is_max, const Abort &ab) {
  const int tid = sy.tid(), lane = tid & 31, warp = tid >> 5;
  const long long ident = is_max ? LLONG_MIN : 0;
  long long v = ident;
  bool ok = true;
  if (tid < 4 * cpg) ok = slot_get(slots + (size_t)tid * 2, v, ab);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    const long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? (u > v ? u : v) : v + u;
  }
  if (lane < 4 && warp < 16) mg_gat[warp * 4 + lane] = v;
  if (sy.any(!ok)) return false;
  if (tid < 4) {
    long long r = ident;
    for (int w = 0; w < (4 * cpg + 31) / 32; ++w) {
      const long long u = mg_gat[w * 4 + tid];
      r = is_max ? (u > r ? u : r) : r + u;
    }
    mg_att[tid] = r;
  }
  sy.sync();
  return true;
}

F5_DEV bool c_attn(const MegaArgs &ma, const MegaAttn &m, const MegaSmem &S, int T, int pos, int &w_sk, int &w_sv,
                   const Abort &ab, uint32_t epoch) {
  const AttnArgs &a = m.a;
  const AttGeo g = att_geo(a, T, pos, gridDim.x, blockIdx.x);
  if (g.kv >= a.nkv) return true;
  const CSync sy;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, hs = tid >> 7, e = tid & 127;
  const int hq = g.kv * 4 + hs;
  const int cm = a.chunk_max;
  uint8_t *scr = S.scr();
  int16_t *q16 = reinterpret_cast<int16_t *>(scr + AT_Q16);
  int16_t *k16n = reinterpret_cast<int16_t *>(scr + AT_K16);
  int16_t *xn = reinterpret_cast<int16_t *>(scr + AT_XN);
  int8_t *k8n = reinterpret_cast<int8_t *>(scr + AT_K8N);
  int8_t *v8n = reinterpret_cast<int8_t *>(scr + AT_V8N);
  const uint8_t *kbuf = scr + AT_K, *vbuf = scr + AT_V;
  const int8_t *kebuf = reinterpret_cast<const int8_t *>(scr + AT_KE);
  const int8_t *vebuf = reinterpret_cast<const int8_t *>(scr + AT_VE);
  long long *sc = reinterpret_cast<long long *>(scr + AT_SC);
  long long *red4 = mg_red;   // [16 warps][4 heads]
  if (!g.ok && blockIdx.x == 0 && tid == 0) atomicOr(a.err, (uint32_t)DERR_KV_FULL);
  const int16_t *cs = a.rope + (size_t)g.pos * 128;
  const size_t kvrow = (size_t)g.kv * a.max_T;
  const bool k_act = hs == 0;

  // ---- 0. every operand in one round of loads: the constants first (their
  // L2 round trip overlaps the wait for the tagged inputs) ----
  const long long qw0 = __ldcg(a.q_norm + e), qw1 = __ldcg(a.q_norm + e + 128);
  const long long kw0 = __ldcg(a.k_norm + e), kw1 = __ldcg(a.k_norm + e + 128);
  const long long cosv = e < a.rot ? __ldcg(cs + e) : 0, sinv = e < a.rot ? __ldcg(cs + 64 + e) : 0;
  const uint32_t itag = (epoch && m.in_tag_op1) ? mk_tag(epoch, m.in_tag_op1) : 0u;
  long long qx0, qx1, kx0 = 0, kx1 = 0, v0 = 0, v1 = 0;
  if (itag) {   // the six tagged words polled together (one L2 round trip per poll)
    const uint32_t *q32 = reinterpret_cast<const uint32_t *>(a.qg16), *k32 = reinterpret_cast<const uint32_t *>(a.k16),
                   *v32 = reinterpret_cast<const uint32_t *>(a.v16);
    const uint32_t *const pw[6] = {q32 + hq * 512 + e, q32 + hq * 512 + e + 128, k32 + g.kv * 256 + e,
                                   k32 + g.kv * 256 + e + 128, v32 + g.kv * 256 + e, v32 + g.kv * 256 + e + 128};
    const bool act[6] = {true, true, k_act, k_act, k_act, k_act};
    uint32_t w6[6];
    ld_tagged_multi<6>(pw, act, itag, w6, ab.flag, ab.err);
    qx0 = tag_s16(w6[0]);
    qx1 = tag_s16(w6[1]);
    if (k_act) {
      kx0 = tag_s16(w6[2]);
      kx1 = tag_s16(w6[3]);
      v0 = tag_s16(w6[4]);
      v1 = tag_s16(w6[5]);
    }
  } else {
    qx0 = __ldcg(a.qg16 + hq * 512 + e);
    qx1 = __ldcg(a.qg16 + hq * 512 + e + 128);
    if (k_act) {
      kx0 = __ldcg(a.k16 + g.kv * 256 + e);
      kx1 = __ldcg(a.k16 + g.kv * 256 + e + 128);
      v0 = __ldcg(a.v16 + g.kv * 256 + e);
      v1 = __ldcg(a.v16 + g.kv * 256 + e + 128);
    }
  }

  // ---- 1. q / k norm + rope; kv_quant of the new k and v ----
  long long kn0, kn1;
  norm_rope_qk(sy, qx0, qx1, qw0, qw1, kx0, kx1, kw0, kw1, cosv, sinv, a.rot, xn, k16n, q16, kn0, kn1, mg_red);
  const unsigned long long mk0 = uabs(kn0) > uabs(kn1) ? uabs(kn0) : uabs(kn1);
  const unsigned long long mv0 = uabs(v0) > uabs(v1) ? uabs(v0) : uabs(v1);
  unsigned long long mk, mv;
  g_max2_ull(sy, mk0, mv0, reinterpret_cast<unsigned long long *>(mg_red), mk, mv);
  const int ek = dynq8_e(mk);
  const int ev = dynq8_e(mv);
  if (k_act) {
    const int8_t k0 = (int8_t)dynq8_apply(kn0, ek), k1 = (int8_t)dynq8_apply(kn1, ek);
    const int8_t w0 = (int8_t)dynq8_apply(v0, ev), w1 = (int8_t)dynq8_apply(v1, ev);
    k8n[e] = k0; k8n[e + 128] = k1;
    v8n[e] = w0; v8n[e + 128] = w1;
    if (g.ok && g.j == 0) {   // append to the cache at slot T (one CTA per KV head)
      const size_t row = (kvrow + T) * 256;
      a.k8[row + e] = k0; a.k8[row + e + 128] = k1;
      a.v8[row + e] = w0; a.v8[row + e + 128] = w1;
      if (e == 0) {
        a.ke[kvrow + T] = (int8_t)(ek - QKV_F);
        a.ve[kvrow + T] = (int8_t)(ev - QKV_F);
      }
    }
  }
  const int ke_new = ek - QKV_F, ve_new = ev - QKV_F;
  sy.sync();
  MG_MARK(2);

  // ---- 2. scores: warp per token, 4 heads at once; lane = 8 dims ----
  int32_t qr[4][8];
#pragma unroll
  for (int h = 0; h < 4; ++h)
#pragma unroll
    for (int i = 0; i < 8; ++i) qr[h][i] = q16[h * 256 + 8 * lane + i];
  long long lmax = LLONG_MIN;   // of head lane >> 3
  const int len = max(0, g.t1 - g.t0);
  const int nfill = (len + MEGA_SUB - 1) / MEGA_SUB;
  bool bad = false;
  for (int si = 0; si < nfill && !bad; ++si) {
    int sb;
    const int n_old = att_fill_rows(g, si, sb);
    const int se = min(sb + MEGA_SUB, g.t1);
    if (n_old > 0) {
      if (si > 0) {
        sy.sync();   // previous fill fully read
        if (tid == 0) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          att_issue(scr + AT_K, scr + AT_KE, a.k8, a.ke, kvrow + sb, n_old, (&mg_bsk));
          mg_cnt[4] += 1;
        }
      }
      const bool got = mwait((&mg_bsk), w_sk & 1, ab);
      ++w_sk;
      if (sy.any(!got)) { bad = true; break; }
    }
    for (int t = sb + warp; t < se; t += MG_CONS) {
      uint2 kw;
      int kex;
      if (t >= g.Told) {   // the new token (t == T)
        kw = *reinterpret_cast<const uint2 *>(k8n + 8 * lane);
        kex = ke_new;
      } else {
        kw = *reinterpret_cast<const uint2 *>(kbuf + (size_t)(t - sb) * 256 + 8 * lane);
        kex = kebuf[t - sb];
      }
      int dot[4] = {0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int b0 = (int)(int8_t)((kw.x >> (8 * j)) & 0xFF), b1 = (int)(int8_t)((kw.y >> (8 * j)) & 0xFF);
#pragma unroll
        for (int h = 0; h < 4; ++h) dot[h] += qr[h][j] * b0 + qr[h][4 + j] * b1;
      }
      // lane group lane >> 3 receives head (lane >> 3)'s total
      const int tot = warp_sum4_i32(dot);
      // rshr(dot * 2048, 15) (SCALE_Q15 = round(2^15/sqrt(256))) is the same
      // rational rounded the same way as rshr(dot, 4); |dot| < 2^30
      const long long s = shift_to(rshr32p(tot, 4), QKV_F - kex - 16);
      lmax = s > lmax ? s : lmax;
      if ((lane & 7) == 0) sc[(lane >> 3) * cm + (t - g.t0)] = s;
    }
  }
  if (sy.any(bad)) return false;
  MG_MARK(3);
  // group score max over the kv head's cpg CTAs (marked slots, phase 0)
  unsigned long long *slots = m.slots + (size_t)g.kv * g.cpg * 8;
  const size_t phase_stride = (size_t)a.nkv * g.cpg * 8;
  if ((lane & 7) == 0) red4[warp * 4 + (lane >> 3)] = lmax;
  sy.sync();
  if (tid < 4) {
    long long mx = LLONG_MIN;
    for (int w = 0; w < MG_CONS; ++w) mx = red4[w * 4 + tid] > mx ? red4[w * 4 + tid] : mx;
    slot_put(slots + (size_t)(g.j * 4 + tid) * 2, mx);
  }
  if (!group_gather(sy, slots, g.cpg, true, ab)) return false;
  MG_MARK(4);

  // ---- 3. exp, group sum, reciprocal, probabilities (Q15) ----
  // one pass over (token, head): thread t works on head t & 3 (MG_CT is a
  // multiple of 4), lanes with equal lane & 3 share a head
  const int hx = tid & 3;
  long long sum = 0;
  {
    const long long mx = mg_att[hx];
    for (int idx = tid; idx < 4 * len; idx += MG_CT) {
      const int i = idx >> 2;
      const long long x = sc[hx * cm + i] - mx;
      const long long es = exp_neg_q(x < 0 ? x : 0);
      sc[hx * cm + i] = es;
      sum += es;
    }
  }
#pragma unroll
  for (int o = 16; o >= 4; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane < 4) red4[warp * 4 + lane] = sum;
  sy.sync();
  if (tid < 4) {
    long long tot = 0;
    for (int w = 0; w < MG_CONS; ++w) tot += red4[w * 4 + tid];
    slot_put(slots + phase_stride + (size_t)(g.j * 4 + tid) * 2, tot);
  }
  if (!group_gather(sy, slots + phase_stride, g.cpg, false, ab)) return false;
  MG_MARK(5);
  if (tid < 4) {
    const long long den = mg_att[tid];
    int64_t rr;
    int re;
    recip_q((uint64_t)(den > 0 ? den : 1), 30, rr, re);
    mg_att[tid] = rr;
    mg_att[4 + tid] = 30 - re + 15;
  }
  sy.sync();
  {
    const long long rcp = mg_att[hx];
    const int psh = (int)mg_att[4 + hx];
    for (int idx = tid; idx < 4 * len; idx += MG_CT) {
      const int i = idx >> 2;
      sc[hx * cm + i] = clip(rshr(sc[hx * cm + i] * rcp, psh), 0, 1 << 15);
    }
  }
  sy.sync();

  // ---- 4. PV: warp = (token phase, head); lane = 8 dims ----
  const int ph = warp >> 2, hv = warp & 3;
  int32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int si = 0; si < nfill && !bad; ++si) {
    int sb;
    const int n_old = att_fill_rows(g, si, sb);
    const int se = min(sb + MEGA_SUB, g.t1);
    if (n_old > 0) {
      if (si > 0) {
        sy.sync();
        if (tid == 0) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          att_issue(scr + AT_V, scr + AT_VE, a.v8, a.ve, kvrow + sb, n_old, (&mg_bsv));
          mg_cnt[5] += 1;
        }
      }
      const bool got = mwait((&mg_bsv), w_sv & 1, ab);
      ++w_sv;
      if (sy.any(!got)) { bad = true; break; }
    }
    for (int t = sb + ph; t < se; t += 4) {
      uint2 vw;
      int vex;
      if (t >= g.Told) {
        vw = *reinterpret_cast<const uint2 *>(v8n + 8 * lane);
        vex = ve_new;
      } else {
        vw = *reinterpret_cast<const uint2 *>(vbuf + (size_t)(t - sb) * 256 + 8 * lane);
        vex = vebuf[t - sb];
      }
      const int32_t p = (int32_t)sc[hv * cm + (t - g.t0)];
      const int sh = 15 - vex - QKV_F;   // in [6, 15]
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[j] += rshr32p(p * (int32_t)(int8_t)((vw.x >> (8 * j)) & 0xFF), sh);
        acc[4 + j] += rshr32p(p * (int32_t)(int8_t)((vw.y >> (8 * j)) & 0xFF), sh);
      }
    }
  }
  if (bad) return false;
  int32_t *pv = reinterpret_cast<int32_t *>(scr + AT_K);   // [4 phases][4 heads][256]; K rows are done
  sy.sync();
#pragma unroll
  for (int j = 0; j < 8; ++j) pv[(ph * 4 + hv) * 256 + 8 * lane + j] = acc[j];
  sy.sync();
  if (len > 0) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int idx = tid + k * MG_CT, h = idx >> 8, dd = idx & 255;
      const int32_t s = pv[h * 256 + dd] + pv[(4 + h) * 256 + dd] + pv[(8 + h) * 256 + dd] + pv[(12 + h) * 256 + dd];
      if (s) atomicAdd(&m.gacc[(g.kv * 4 + h) * 256 + dd], s);
    }
  }
  MG_MARK(6);
  release_scratch(sy, (&mg_bfree));
  return true;
}

// ---------------------------------------------------------------------------
F5_DEV void c_begin(const MegaArgs &ma, const MegaBegin &B, int tok, uint32_t epoch) {
  const int tid = threadIdx.x, G = gridDim.x, b = blockIdx.x;
  if (tok < 0 || tok >= B.vocab) {
    if (b == 0 && tid == 0) atomicOr(ma.err, DERR_RANGE);
    tok = 0;
  }
  if (B.x16t) {
    // tagged residual, the whole vector on every GPU (tagged as op 0); the
    // CTA's own residual rows -- the rows its residual epilogues own: this
    // rank's share, partitioned over the CTAs -- are also kept in mg_xres
    const int16_t *src = B.emb + (size_t)tok * B.H;
    const uint32_t tag = mk_tag(epoch, 1);
    for (int i = part_lo(B.H, G, b) + tid; i < part_lo(B.H, G, b + 1); i += MG_CT) B.x16t[i] = tag_word(tag, src[i]);
    const int r0 = B.res_row0 + part_lo(B.res_rows, G, b), r1 = B.res_row0 + part_lo(B.res_rows, G, b + 1);
    for (int i = r0 + tid; i < r1 && i - r0 < MG_XRES; i += MG_CT) mg_xres[i - r0] = src[i];
  } else {
    const uint4 *src = reinterpret_cast<const uint4 *>(B.emb + (size_t)tok * B.H);
    uint4 *dst = reinterpret_cast<uint4 *>(B.x16);
    for (int i = b * MG_CT + tid; i < B.H / 8; i += G * MG_CT) dst[i] = src[i];
  }
  for (int i = b * MG_CT + tid; i < B.zero_n; i += G * MG_CT) B.zero[i] = make_uint4(0, 0, 0, 0);
  if (b == 0 && tid == 0) *B.key = 0ull;
}

// descriptor of op `oi` into cop[oi & 1]: cp.async by the first threads,
// completed (cp.async.wait_all) before the next group barrier publishes it
constexpr int MG_DESC_V4 = (int)(sizeof(MegaOp) / 16);
static_assert(MG_DESC_V4 <= MG_CT, "descriptor copy: one 16-byte piece per thread");
F5_DEV void stage_desc(const MegaArgs &ma, const MegaSmem &S, int oi) {
  const int t = threadIdx.x;
  if (t < MG_DESC_V4) {
    const uint32_t dst = smem_u32(reinterpret_cast<uint4 *>(&mg_cop[oi & 1]) + t);
    const uint4 *src = reinterpret_cast<const uint4 *>(ma.ops + oi) + t;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
}
F5_DEV void stage_wait() {
  if (threadIdx.x < MG_DESC_V4) asm volatile("cp.async.wait_all;" ::: "memory");
}

F5_DEV void consumers(const MegaArgs &ma, const MegaSmem &S, int tok, int T, int pos, const Abort &ab,
                      uint32_t epoch) {
  const CSync sy;
  RingPos rp;
  int w_sd = 0, w_sk = 0, w_sv = 0, w_g = 0;
  unsigned long long *tr = F5_MEGA_TRACE && ma.trace ? ma.trace + (size_t)blockIdx.x * ma.nops * MEGA_TRACE_SLOTS : nullptr;
  stage_desc(ma, S, 0);
  for (int oi = 0; oi < ma.nops; ++oi) {
    // The sync publishes op oi's staged descriptor and retires every reader
    // of the buffer staged next.  Ops whose inputs are dataflow-tagged need
    // no grid barrier: their loads wait for the words themselves.
    stage_wait();
    if (oi > 0 && tr && threadIdx.x == 0) tr[(size_t)(oi - 1) * MEGA_TRACE_SLOTS + 7] = gtimer();   // arrival
    sy.sync();
    const int bar = mg_cop[oi & 1].bar;
    if (bar >= 0 && !counter_barrier(sy, &ma.bars[bar], gridDim.x, ab)) return;
#if F5_MEGA_TRACE
    if (threadIdx.x == 0) mg_tr = tr ? tr + (size_t)oi * MEGA_TRACE_SLOTS : nullptr;
#endif
    if (oi + 1 < ma.nops) stage_desc(ma, S, oi + 1);
    const MegaOp &op = mg_cop[oi & 1];
    if (tr && threadIdx.x == 0) tr[(size_t)oi * MEGA_TRACE_SLOTS] = gtimer();
    bool ok = true;
    switch (op.kind) {
      case MK_BEGIN: c_begin(ma, op.b, tok, epoch); break;
      case MK_GEMV:
        ok = op.g.K > 4096 ? c_gemv_split<3>(op.g, S, rp, ab, epoch) : c_gemv4096(op.g, S, rp, ab, epoch, w_g, T);
        break;
      case MK_DN: ok = c_dn(ma, op.d, S, w_sd, ab, epoch); break;
      case MK_ATTN: ok = c_attn(ma, op.at, S, T, pos, w_sk, w_sv, ab, epoch); break;
      default: break;
    }
    if (tr && threadIdx.x == 0) tr[(size_t)oi * MEGA_TRACE_SLOTS + 1] = gtimer();
    if (!ok) {
      stage_wait();
      return;
    }
  }
}

#if F5_MEGA_TRACE
#define F5_MEGA_KERNEL k_mega_traced
#else
#define F5_MEGA_KERNEL k_mega
#endif
__global__ void __launch_bounds__(MEGA_THREADS, 1) F5_MEGA_KERNEL(const __grid_constant__ MegaArgs ma) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ns = ma.ns;
  MegaSmem S;
  S.ns = ns;
  const Abort ab = {ma.bars + ma.nbars - 2, ma.err};

  if (tid == 0) {
    for (int i = 0; i < ns; ++i) {
      mbar_init(&mg_full[i], 1);
      mbar_init(&mg_empty[i], MG_CONS);
    }
    mbar_init(&mg_bsd, 1);
    mbar_init(&mg_bsk, 1);
    mbar_init(&mg_bsv, 1);
    mbar_init(&mg_bfree, 1);
    mbar_init(&mg_bpd[0], 1);
    mbar_init(&mg_bpd[1], 1);
    mbar_init(&mg_gfull, 1);
    mbar_init(&mg_gfree, 1);
    for (int i = 0; i < 7; ++i) mg_cnt[i] = 0;
    mg_abort = 0;
    mg_last = 0;
#if F5_MEGA_TRACE
    mg_tr = nullptr;
#endif
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < F5_LUT_RSQRT_N; i += MEGA_THREADS) mg_lut_rsqrt[i] = f5_lut_rsqrt[i];
  for (int i = tid; i < F5_LUT_RECIP_N; i += MEGA_THREADS) mg_lut_recip[i] = f5_lut_recip[i];
  for (int i = tid; i < F5_LUT_EXP2_N; i += MEGA_THREADS) mg_lut_exp2[i] = f5_lut_exp2[i];
  for (int i = tid; i < F5_LUT_SIGMOID_N; i += MEGA_THREADS) mg_lut_sigmoid[i] = f5_lut_sigmoid[i];
  for (int i = tid; i < F5_LUT_SOFTPLUS_N; i += MEGA_THREADS) mg_lut_softplus[i] = f5_lut_softplus[i];
  // step parameters: written by the host or by the previous launch only
  const volatile StepParams *vp = ma.params;
  const int tok = vp->tok, T = vp->T, pos = vp->pos;
  const uint32_t epoch = mega_epoch(vp->launch);
  __syncthreads();

  if (warp == MG_CONS) {
    if (lane == 0) producer(ma, S, T, pos, ab);
  } else if (warp < MG_CONS) {
    consumers(ma, S, tok, T, pos, ab, epoch);
  }
  __syncwarp();   // reconverge each warp (the producer lane joins its warp) before the CTA barrier
  __syncthreads();

  if (tid == 0) {
    // never exit with a bulk copy in flight: wait (bounded) for the last
    // issued phase of every barrier; a completed phase returns at once
    const int issued = mg_cnt[0];
    for (int s = 0; s < ns && s < issued; ++s) {
      const int last = issued - 1 - ((issued - 1 - s) % ns);   // last chunk that used stage s
      mbar_wait(&mg_full[s], (last / ns) & 1, MG_WAIT_NS);
    }
    if (mg_cnt[1]) mbar_wait(&mg_bsd, (mg_cnt[1] - 1) & 1, MG_WAIT_NS);
    if (mg_cnt[6]) mbar_wait(&mg_gfull, (mg_cnt[6] - 1) & 1, MG_WAIT_NS);
    const int nk = mg_cnt[2] + mg_cnt[4], nv = mg_cnt[3] + mg_cnt[5];
    if (nk) mbar_wait(&mg_bsk, (nk - 1) & 1, MG_WAIT_NS);
    if (nv) mbar_wait(&mg_bsv, (nv - 1) & 1, MG_WAIT_NS);
    __threadfence();
    mg_last = atomicAdd(&ma.bars[ma.nbars - 1], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!mg_last) return;
  __threadfence();
  if (tid == 0) {
    // step end (ref/gen_model_script.py:641 argmax, first max wins)
    StepParams *p = ma.params;
    unsigned long long k = __ldcg(ma.ops[ma.nops - 1].g.argmax_key);
    bool aborted = __ldcg(ma.bars + ma.nbars - 2) != 0;
    if (ma.nrank > 1) {
      // vocab-sharded head: publish this rank's key to every rank (two words
      // {half, marker = launch + 1}), then combine all ranks' keys; the
      // global row index is in the key, so max over ranks = the first max
      const unsigned long long mk = (unsigned long long)(uint32_t)(vp->launch + 1) << 32;
      for (int r = 0; r < ma.nrank; ++r) {
        unsigned long long *d = reinterpret_cast<unsigned long long *>(
            reinterpret_cast<char *>(ma.xkey + 2 * ma.rank) + ma.peer_delta[r]);
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(d), "l"(mk | (k & 0xFFFFFFFFull)) : "memory");
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(d + 1), "l"(mk | (k >> 32)) : "memory");
      }
      unsigned long long best = 0ull, t0 = 0;
      for (int r = 0; r < ma.nrank && !aborted; ++r) {
        for (uint32_t it = 0;; ++it) {
          unsigned long long lo, hi;
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(lo) : "l"(ma.xkey + 2 * r) : "memory");
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(hi) : "l"(ma.xkey + 2 * r + 1) : "memory");
          if ((lo & ~0xFFFFFFFFull) == mk && (hi & ~0xFFFFFFFFull) == mk) {
            const unsigned long long kr = (hi << 32) | (lo & 0xFFFFFFFFull);
            best = kr > best ? kr : best;
            break;
          }
          const unsigned long long t = gtimer();
          if (t0 == 0) t0 = t;
          else if (t - t0 > MG_WAIT_NS) {
            atomicOr(ma.err, DERR_TIMEOUT);
            aborted = true;
            break;
          }
        }
      }
      k = best;
    }
    const int row = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    p->next_tok = row;
    p->max_val = (int)((uint32_t)(k >> 32) ^ 0x80000000u);
    p->err |= __ldcg(ma.err);
    if (ma.advance && !aborted) {
      p->tok = row;
      p->pos += 1;
      p->T += 1;
      p->steps += 1;
    }
    p->launch += 1;
  }
  {   // the plain residual for readers outside the step (tagged words -> int16)
    const MegaBegin &B = ma.ops[0].b;
    if (B.x16t)
      for (int i = tid; i < B.H; i += MEGA_THREADS) B.x16[i] = (int16_t)tag_s16(__ldcg(B.x16t + i));
  }
  __syncthreads();
  for (int i = tid; i < ma.nbars; i += MEGA_THREADS) ma.bars[i] = 0u;
}

#if !F5_MEGA_TRACE
static size_t mega_smem_bytes(int ns, int chunk_max) {
  size_t scr = (size_t)AT_SC + (size_t)4 * chunk_max * 8;
  if (scr < (size_t)DN_END) scr = DN_END;
  return (size_t)ns * MEGA_STAGE + MG_XS + MG_RESB + MG_GAINB + scr;
}

cudaError_t mega_config(int chunk_max, int *grid, size_t *smem, int *ns) {
  int dev = 0, sms = 0, optin = 0, coop = 0;
  cudaError_t e;
  if ((e = cudaGetDevice(&dev))) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))) return e;
  if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev))) return e;
  if ((e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev))) return e;
  if (!coop) return cudaErrorNotSupported;
  cudaFuncAttributes fa;
  if ((e = cudaFuncGetAttributes(&fa, k_mega))) return e;
  int n = MG_NS_MAX;
  while (n >= 3 && mega_smem_bytes(n, chunk_max) + fa.sharedSizeBytes > (size_t)optin) --n;
  if (n < 3) return cudaErrorInvalidValue;
  const size_t bytes = mega_smem_bytes(n, chunk_max);
  // the limit is a property of the kernel, shared by every context of the
  // process: raise it to what any configuration may use, never lower it
  // below another context's launch size
  if ((e = cudaFuncSetAttribute(k_mega, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)((size_t)optin - fa.sharedSizeBytes))))
    return e;
  int per_sm = 0;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_mega, MEGA_THREADS, bytes))) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  *grid = sms;   // one CTA per SM (the kernel is written for exactly one)
  *smem = bytes;
  *ns = n;
  return cudaSuccess;
}

cudaError_t launch_mega(const MegaArgs &a, int grid, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(MEGA_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_mega, a);
}

#else
// The traced instance: same grid, shared memory and cooperative launch as
// the step kernel (its dynamic shared-memory limit raised on each call:
// tracing is a diagnostic, and the limit is per device).
cudaError_t launch_mega_traced(const MegaArgs &a, int grid, size_t smem, cudaStream_t st) {
  int dev = 0, optin = 0;
  cudaFuncAttributes fa;
  cudaError_t e;
  if ((e = cudaGetDevice(&dev))) return e;
  if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev))) return e;
  if ((e = cudaFuncGetAttributes(&fa, k_mega_traced))) return e;
  if (smem + fa.sharedSizeBytes > (size_t)optin) return cudaErrorInvalidValue;
  if ((e = cudaFuncSetAttribute(k_mega_traced, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)((size_t)optin - fa.sharedSizeBytes))))
    return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(MEGA_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_mega_traced, a);
}
#endif

}  // namespace f5
