// step.cu — the persistent decode-step kernel.
//
// Reference: the device branch of ForwardToken / ForwardLayerDevice
// (src/forward.cc:700-794), which issues, per layer, RMSNorm, three
// projections, RoPE, a KV-cache write, attention, wo, a residual add,
// RMSNorm, gate/up, SiLU*mul, down and a residual add as separate kernels with
// device synchronisation in between.
//
// Here one cooperative launch of one CTA per SM (16 warps each) runs the
// whole step as a list of phases: per layer the fused QKV projection (RMSNorm
// prologue; bias, RoPE, q store, K/V cache write epilogue), attention, wo
// (residual epilogue), fused gate/up (RMSNorm prologue, SiLU*mul epilogue),
// down (residual epilogue); then the lm_head (final RMSNorm, logits, greedy
// argmax) and the token/position update. The embedding row is read in place.
//
// Phases are separated by grid barriers, but the weight stream is not: every
// warp owns a ring of shared-memory slots fed by cp.async.bulk, and its
// producer walks the warp's super-blocks of ALL projection phases in order.
// A slot freed in phase p is refilled with the next super-block the warp will
// need, which may belong to phase p + 1 or later, so HBM keeps streaming
// weights while the CTA waits at a barrier, stages activations or runs
// attention. The arithmetic is the standalone GEMV's (gemv_dev.cuh), so
// results are identical to the per-op path.
//
// Attention cuts each KV head's positions into G / KV equal slices, one slice
// per CTA, so every CTA carries at most one piece of work. A CTA's 16 warps
// take blocks of positions round robin, each keeping an online softmax
// (m, l, o) per query head of the GQA group; the CTA combines its warps in
// warp order. A slice that is a whole head writes the output; otherwise it
// leaves (m, l, o) in a workspace record and the last slice of the head to
// arrive combines the slices in position order. Deterministic, like the GEMV
// fix-ups.
//
// Every wait is bounded (about 2 s of clock64 polling): on timeout the kernel
// records MLB_ERR_TIMEOUT in the status word, waits (bounded) for its own
// bulk copies still in flight and returns; other CTAs see the status word at
// their next barrier and return too. A launch that finds the status word set
// does nothing.
#include "step.cuh"

#include <algorithm>
#include <cstring>

#include "gemv_dev.cuh"

namespace mlb {

namespace {

constexpr int kStepWarps = kGemvWarps;  // 16
constexpr int kStepThreads = kStepWarps * 32;
constexpr int kMaxGrid = 256;
constexpr long long kWaitCycles = 4000000000LL;

// HG: query heads per pass over the positions (1, 2 or 4; groups of other
// sizes run ceil(gq / HG) passes with the missing heads masked).
template <int HG>
struct AttnShape {
  static constexpr int PB = 4;                // positions per warp block
  static constexpr int NV = HG * PB;          // scores per block (<= 16)
};

// A softmax record (m, l, o[D]) is kRec(D) floats with o at offset kRecO, so
// that o starts on a 16-byte boundary (D is a multiple of 4).
constexpr int kRecO = 4;
__host__ __device__ constexpr int attn_rec(int D) { return D + kRecO; }


// Residual rows a CTA prefetches into shared memory for its residual epilogue
// (16 tiles; larger ranges read the residual from L2 in the epilogue).
constexpr int kResidPre = 256;

// A warp's weight-stream producer: its walk over runs (lane 0's, in shared
// memory; see producer_seek).
struct Producer {
  int p;       // phase of the next run (nphases: none left)
  int seg;     // segment of the CTA range (one per chunk group)
  int sbase;   // its first super-block, relative to the range start
  int tw, Tw;  // the window: first tile (segment-relative), tile count
  int c;       // chunk: the run is chunk c of the window's Tw tiles
};

// The producer's current run in registers (lane 0's): `left` super-blocks
// more, `next` the next one's address, `step` bytes between them (one tile).
struct ProducerRun {
  const uint8_t* next;
  int step, left;
};

// Shared state of one CTA besides the ring and the scratch region.
struct StepShared {
  StepPhase cur[2];  // this phase's descriptor and the next one's (prefetched)
  // the launch arguments, copied once: the phases read them from here rather
  // than through a generic pointer to the parameter space
  StepArgs args;
  float inv_rms[4];
  float part[kStepWarps];
  int run_u0[kWinRuns + 1];
  int run_t[kWinRuns], run_grp[kWinRuns], run_cc0[kWinRuns];
  int nruns;
  int flag;
  unsigned int tp_gen0;  // exchange steps completed before this decode step
  unsigned int tp_kgen0; // decode steps completed before this one
  int tp_fail;           // a tagged read gave up
  int pos, token;        // the step's position and input token (read once)
  Producer prod[kStepWarps];  // each warp's producer (lane 0 reads and writes it)
  alignas(16) float resid_pre[kResidPre];  // residual rows of this CTA's tiles (epilogue)
  alignas(16) float2 rope_pre[64];         // the position's rope row (QKV epilogue, D <= 128)
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void record_error(DeviceStatus* st, int code, int where) {
  if (atomicCAS(&st->code, 0, code) == 0) atomicExch(&st->where, where);
}

// Grid barrier over all CTAs of the launch (co-resident: cooperative launch).
// Barrier k of a step waits for the arrival counter to reach k * gridDim.x:
// each CTA arrives with a fire-and-forget release add (after bar.sync, so it
// publishes the whole CTA's writes) and knows the target from its own count
// of barriers; the poll is an acquire load followed by bar.sync. The step's
// last CTA resets the counter.
// Returns false (block-uniform) when the wait timed out or another CTA
// recorded an error.
__device__ bool grid_barrier(unsigned int* counter, unsigned int k, DeviceStatus* st, int where,
                             int* flag, long long limit = kWaitCycles) {
  __syncthreads();  // the CTA's writes happen before thread 0's release below
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
    const unsigned int target = k * gridDim.x;
    const long long t0 = clock64();
    int ok = 1;
    while ((int)(ld_acquire_u32(counter) - target) < 0) {
      if (*(volatile int*)&st->code != 0) {
        ok = 0;
        break;
      }
      if (clock64() - t0 > limit) {
        record_error(st, MLB_ERR_TIMEOUT, where);
        ok = 0;
        break;
      }
    }
    *flag = ok;  // the acquire load above orders the CTA's later reads (bar.sync)
  }
  __syncthreads();
  const int ok = *flag;
  __syncthreads();
  return ok != 0;
}

__device__ __forceinline__ void red_release_sys_add(unsigned int* p, unsigned int v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_relaxed_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Tensor parallel, one thread: wait (bounded) until c[r] >= target for every
// rank r other than this one (skip: include this rank too), polling relaxed
// and acquiring once at the end. Returns false on timeout or a recorded error.
__device__ __forceinline__ bool tp_wait_all(const TpXchg* x, long long off, unsigned int target,
                                            bool include_self, DeviceStatus* st, int where) {
  const unsigned int* c = reinterpret_cast<const unsigned int*>(x->peers[x->me] + off);
  const long long t0 = clock64();
  for (int r = 0; r < x->n; ++r) {
    if (r == x->me && !include_self) continue;
    while ((int)(ld_relaxed_sys_u32(c + r) - target) < 0) {
      if (*(volatile int*)&st->code != 0) return false;
      if (clock64() - t0 > kWaitCycles) {
        record_error(st, MLB_ERR_TIMEOUT, where);
        return false;
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  return true;
}

// ------------------------------------------------------------ weight ring

// Per-warp ring of `stages` slots. Lane 0 issues copies; every lane tracks the
// consumer position (slot, parity) identically.
struct Ring {
  uint8_t* base;     // this warp's slots
  uint64_t* bars;    // this warp's barriers
  int stride, stages;
  int slot;
  uint32_t parity;
  int inflight;      // copies issued and not yet consumed (lane 0's count)
};

// Tiles in the window of a segment that starts `rem` tiles before the end of
// the segment: whole tiles, at most kWinRuns of them and at most win_sbs
// super-blocks (the producer and the consumer use the same rule).
__device__ __forceinline__ int win_tiles(int rem, int nc) {
  return max(1, min(min(rem, kWinRuns), win_sbs<1>() / nc));
}

// The producer side (lane 0's): the next super-block this warp will need,
// over all projection phases in order. The CTA's per-phase ranges come from
// its table in shared memory (attention phases have empty ranges), so
// crossing into the next phase costs no global load. Each segment of a range
// (one chunk group) runs chunk-major: in each window of tiles, warp w takes
// chunk w of every tile, then chunk w + 16, ... A run (one chunk of a
// window's tiles) is a pointer walk held in registers; the walk over runs is
// kept in shared memory (Producer).

// Lane 0: the first segment from pr.seg on in which this warp has chunks;
// false when none is left in the phase.
__device__ __forceinline__ bool producer_segment(Producer& pr, const StepCta& e, int warp) {
  for (; pr.seg < e.nseg; ++pr.seg) {
    const int nc = e.nc[pr.seg], T = e.T[pr.seg];
    if (warp < nc && T > 0) {
      pr.sbase = pr.seg == 0 ? 0 : e.T[0] * e.nc[0];
      pr.tw = 0;
      pr.Tw = win_tiles(T, nc);
      pr.c = warp;
      return true;
    }
  }
  return false;
}

// Lane 0: from phase pr.p on, the first phase with super-blocks for this warp.
__device__ __forceinline__ void producer_seek(Producer& pr, const StepCta* tab, int nph,
                                              int warp) {
  while (pr.p < nph) {
    pr.seg = 0;
    if (producer_segment(pr, tab[pr.p], warp)) return;
    pr.p = tab[pr.p].next;
  }
}

// Lane 0: the run at the producer's position.
__device__ __forceinline__ ProducerRun producer_load_run(const Producer& pr, const StepCta* tab,
                                                         int nph, int sbb) {
  ProducerRun run{nullptr, 0, 0};
  if (pr.p >= nph) return run;
  const StepCta& e = tab[pr.p];
  const int nc = e.nc[pr.seg];
  run.next = e.w + ((size_t)pr.sbase + (size_t)pr.tw * nc + pr.c) * sbb;
  run.step = nc * sbb;
  run.left = pr.Tw;
  return run;
}

// Lane 0: the next run: the warp's next chunk of the window, else the next
// window, segment or phase (out of line: once per run).
__device__ __noinline__ ProducerRun producer_next_run(Producer& pr, const StepCta* tab, int nph,
                                                      int warp, int sbb) {
  const StepCta& e = tab[pr.p];
  const int nc = e.nc[pr.seg];
  pr.c += kStepWarps;
  if (pr.c >= nc) {
    pr.c = warp;
    pr.tw += pr.Tw;
    if (pr.tw < e.T[pr.seg]) {
      pr.Tw = win_tiles(e.T[pr.seg] - pr.tw, nc);
    } else {
      ++pr.seg;  // segment done: the next one, else the next phase
      if (!producer_segment(pr, e, warp)) {
        pr.p = e.next;
        producer_seek(pr, tab, nph, warp);
      }
    }
  }
  return producer_load_run(pr, tab, nph, sbb);
}

// Lane 0: the producer's next super-block into ring slot `slot`, if any is left.
__device__ __forceinline__ void producer_issue(Producer& pr, ProducerRun& run, Ring& rg,
                                               int slot, const StepCta* tab, int nph, int warp,
                                               int sbb) {
  if (run.left <= 0) return;
  uint64_t* bar = rg.bars + slot;
  mbar_arrive_expect_tx(bar, sbb);
  bulk_g2s(rg.base + (size_t)slot * rg.stride, run.next, sbb, bar);
  ++rg.inflight;
  run.next += run.step;
  if (--run.left == 0) run = producer_next_run(pr, tab, nph, warp, sbb);
}

struct StepRefill {
  Producer* pr;
  ProducerRun* run;
  Ring* rg;
  const StepCta* tab;
  int nph, warp, sbb;
  __device__ __forceinline__ void operator()(int slot) {
    producer_issue(*pr, *run, *rg, slot, tab, nph, warp, sbb);
  }
};

// ----------------------------------------------------------- GEMV phase

struct GemvScratch {
  uint32_t* frag;
  float* side;
  float* parts;
  float* red;
};

template <int QT>
__device__ __forceinline__ GemvScratch gemv_scratch(uint8_t* scratch, const StepGemv& g) {
  const int nslots = g.ngroups > 1 ? 2 : 1;
  GemvScratch s;
  s.frag = reinterpret_cast<uint32_t*>(scratch);
  s.side = reinterpret_cast<float*>(s.frag + (size_t)nslots * g.gc * frag_chunk_u32<1>());
  s.parts = s.side + (size_t)nslots * g.gc * side_per_chunk<QT, 1>();
  s.red = s.parts + (size_t)win_sbs<1>() * 16;
  return s;
}

// One warp: the RMSNorm factor 1 / sqrt(mean x^2 + eps) from the producing
// phase's n per-tile sums of squares, summed in one fixed order and broadcast
// from lane 0, so every warp of every CTA gets the same bits. Eight
// independent loads per lane per round (one L2 round trip up to 256 tiles).
// Plain (L1-cached) loads: every warp of every CTA reads the same n values,
// written by other CTAs before the grid barrier whose acquire orders these
// reads, so the CTA's warps share its L1 lines instead of each sending the
// same requests to the few L2 lines that hold them.
__device__ __forceinline__ float warp_inv_rms(const float* ss, int n, int k, float eps) {
  const int lane = threadIdx.x & 31;
  float v = 0.0f;
  for (int i0 = 0; i0 < n; i0 += 256) {
    float t[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int i = i0 + lane + 32 * q;
      t[q] = i < n ? ss[i] : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) v += t[q];
  }
  v = __shfl_sync(0xffffffffu, warp_sum(v), 0);
  const float t = __fdiv_rn(v, (float)k);
  return __fdiv_rn(1.0f, sqrtf(__fadd_rn(t, eps)));
}

// One warp: in each segment of the CTA range, its chunks (warp, warp + 16,
// ... of the segment's group) of x, times the RMSNorm factor (from ss) and the
// norm weight when norm_w is set, into the group's B fragments and side data
// (the same arithmetic as stage_x_m1). Inputs past k stage as zero.
template <int QT>
__device__ __forceinline__ void stage_chunks_warp(const float* x, int k, const float* norm_w,
                                                  const float* ss, int ss_n, float eps,
                                                  const StepCta& ct, int gc, uint32_t* frag,
                                                  float* side) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int SPC = side_per_chunk<QT, 1>();
  float inv = 1.0f;
  bool have_inv = norm_w == nullptr;
  for (int seg = 0; seg < ct.nseg; ++seg) {
    const int slot0 = (ct.grp[seg] - ct.grp[0]) * gc;  // staged chunk of the group's chunk 0
    for (int cc = warp; cc < ct.nc[seg]; cc += kStepWarps) {
      const int kc = (ct.grp[seg] * gc + cc) * kChunkK;  // first input of the chunk
      float4 v[2], w[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // quads lane and lane + 32 of the chunk
        const int k0 = kc + (lane + 32 * h) * 4;
        v[h] = load_quad(x, k0, k, false);
        w[h] = norm_w ? load_quad(norm_w, k0, k, true) : make_float4(1.f, 1.f, 1.f, 1.f);
      }
      if (!have_inv) {  // its loads overlap the ones above
        inv = warp_inv_rms(ss, ss_n, k, eps);
        have_inv = true;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int q4 = lane + 32 * h;
        float e[4] = {v[h].x, v[h].y, v[h].z, v[h].w};
        if (norm_w) {
          const float wv[4] = {w[h].x, w[h].y, w[h].z, w[h].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) e[i] = __fmul_rn(__fmul_rn(e[i], inv), wv[i]);
        }
        const float corr = block_sum8(
            stage_quad<QT, 1>(frag + (size_t)(slot0 + cc) * frag_chunk_u32<1>(), 0, q4, e));
        float* sd = side + (size_t)(slot0 + cc) * SPC;
        if ((q4 & 7) == 0) sd[q4 >> 3] = corr;
        if (QT == MLB_Q4_1) {
          const float s4 = block_sum8((e[0] + e[1]) + (e[2] + e[3]));
          if ((q4 & 7) == 0) sd[8 + (q4 >> 3)] = s4;
        }
      }
    }
  }
}


// One warp, one chunk-major window of Tw tiles: chunk c = warp, warp + 16, ...
// of every tile, from the ring in the producer's order; each super-block's
// partial goes to its window-relative index j nc + c. Returns false (warp-
// uniform) when a wait gave up.
template <int QT>
__device__ __forceinline__ bool consume_chunks(int Tw, int nc, const uint32_t* frag,
                                               const float* side, float* parts, Ring& rg,
                                               StepRefill& refill, DeviceStatus* status,
                                               int where) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int fl = lane < 8 ? lane : (lane & 7);  // lanes past the B columns: any valid data
  constexpr int SPC = side_per_chunk<QT, 1>();
  for (int c = warp; c < nc; c += kStepWarps) {
    uint32_t B[16][2];
    load_b(frag + (size_t)c * frag_chunk_u32<1>() + fl * kFragLaneStride, B);
    const float* sd = side + (size_t)c * SPC;
    for (int j = 0; j < Tw; ++j) {
      uint64_t* bar = rg.bars + rg.slot;
      if (!mbar_try_wait(bar, rg.parity) && !mbar_wait_bounded(bar, rg.parity, status, where))
        return false;
      float acc0 = 0.0f, acc1 = 0.0f;
      sb_accumulate<QT, 1>(rg.base + (size_t)rg.slot * rg.stride, lane, B, sd, acc0, acc1);
      store_sb_partial<1>(parts, j * nc + c, lane, acc0, acc1);
      // every lane has read the slot; lane 0 reuses it for the stream's next
      // super-block (the mbarrier orders the copy after the reads)
      __syncwarp();
      if (lane == 0) {
        --rg.inflight;
        refill(rg.slot);
      }
      if (++rg.slot == rg.stages) {
        rg.slot = 0;
        rg.parity ^= 1u;
      }
    }
  }
  return true;
}

// Returns false (block-uniform) when a wait failed; the caller drains and exits.
template <int QT>
__device__ bool gemv_phase(StepShared& sh, StepPhase& cur, const StepCta& ct, uint8_t* scratch,
                           Ring& rg, Producer& pr, ProducerRun& run, const StepCta* tab,
                           const StepArgs& a) {
  const StepGemv& g = cur.g;
  const int warp = threadIdx.x >> 5;
  const int cb = ct.cb, ce = ct.ce;
  const float* x = g.x ? g.x : a.embedding + (size_t)sh.token * a.dim;
  if (g.tp_ar >= 0 && threadIdx.x == 0)  // this phase's exchange step tag (read after syncs)
    cur.g.epi.tp_tag = sh.tp_gen0 + (unsigned int)g.tp_ar + 1u;
  if (cb >= ce) return true;
  const GemvScratch sc = gemv_scratch<QT>(scratch, g);
  const int g0 = ct.grp[0], g1 = ct.grp[ct.nseg - 1];
  // Every warp needs only its own chunks of x: it stages them itself and
  // starts at once (the RMSNorm statistic, when there is one, from the
  // producing phase's per-tile sums of squares). Otherwise (the statistic of
  // the embedding row) the block stages all of x first.
  if (g.norm_w == nullptr || g.ss_in != nullptr) {
    stage_chunks_warp<QT>(x, g.k, g.norm_w, g.ss_in, g.ss_n, g.eps, ct, g.gc, sc.frag, sc.side);
    __syncwarp();
  } else {
    stage_x_m1<QT>(x, g.k, g.norm_w, g.eps, g.gc, g.nchunks, g0, g1, sc.frag, sc.side, sh.part,
                   sh.inv_rms);
    __syncthreads();
  }
  // residual of the first layer: the embedding row (patched before the
  // barrier below, read only after it)
  if (threadIdx.x == 0 && g.epi.kind == kEpiResidual && g.epi.resid == nullptr)
    cur.g.epi.resid = a.embedding + (size_t)sh.token * a.dim;
  // Epilogue inputs fetched now, so the epilogue after the weight stream does
  // not wait on L2: the residual rows of a one-segment range (cp.async into
  // shared memory, complete before the barrier ahead of finish_runs), and the
  // position from shared memory.
  if (g.epi.kind == kEpiResidual && ct.nseg == 1 && g.ngroups == 1) {
    const int t0 = ct.t0[0], nt = ct.T[0];
    if (nt * 16 <= kResidPre && (t0 + nt) * 16 <= g.epi.n_out) {
      const float* rs = g.epi.resid ? g.epi.resid : a.embedding + (size_t)sh.token * a.dim;
      for (int i = threadIdx.x; i < nt * 4; i += blockDim.x)
        cp_async16(sh.resid_pre + i * 4, rs + (size_t)t0 * 16 + i * 4);
      cp_async_commit();
      if (threadIdx.x == 0) {
        cur.g.epi.resid_s = sh.resid_pre;
        cur.g.epi.resid_t0 = t0;
      }
    }
  }
  if (g.epi.kind == kEpiQkv) {
    // the rope row of this position, fetched now for the epilogue
    const int D = g.epi.head_dim;
    const float2* src = g.epi.rope + (size_t)sh.pos * (D / 2);
    for (int i = threadIdx.x; i < D / 4; i += blockDim.x)
      cp_async16(reinterpret_cast<float4*>(sh.rope_pre) + i, reinterpret_cast<const float4*>(src) + i);
    cp_async_commit();
    if (threadIdx.x == 0) {
      cur.g.epi.pos_set = 1;
      cur.g.epi.pos_now = sh.pos;
      cur.g.epi.rope_s = sh.rope_pre;
    }
  }
  const EpiParams& epi = cur.g.epi;
  RunTable rt{sh.run_u0, sh.run_t, sh.run_grp, sh.run_cc0};
  const FinishGeom fg{g.ntiles, g.nchunks, g.gc, g.ngroups, 1};
  StepRefill refill{&pr, &run, &rg, tab, a.nphases, warp, a.sb_stride};
  constexpr int SPC = side_per_chunk<QT, 1>();

  // Each segment in chunk-major windows of whole tiles (the producer walks
  // the same order).
  int sbase = cb;
  for (int seg = 0; seg < ct.nseg; ++seg) {
    const int nc = ct.nc[seg], T = ct.T[seg], grp = ct.grp[seg];
    const int slot0 = (grp - g0) * g.gc;
    for (int tw = 0; tw < T;) {
      const int Tw = win_tiles(T - tw, nc);
      const int wb = sbase + tw * nc;
      if (!consume_chunks<QT>(Tw, nc, sc.frag + (size_t)slot0 * frag_chunk_u32<1>(),
                              sc.side + (size_t)slot0 * SPC, sc.parts, rg, refill, a.status, 20))
        sh.flag = 0;  // set to 1 at the phase start; every writer stores 0
      // run r of the window is tile t0 + tw + r of the group (read by
      // finish_runs after the barrier)
      for (int r = threadIdx.x; r <= Tw; r += blockDim.x) {
        rt.u0[r] = wb + r * nc;
        if (r < Tw) {
          rt.t[r] = ct.t0[seg] + tw + r;
          rt.grp[r] = grp;
          rt.cc0[r] = 0;
        }
      }
      cp_async_wait_all();  // this thread's prefetched residual rows have landed
      __syncthreads();
      if (!sh.flag) return false;  // block-uniform: read after the barrier
      finish_runs<1>(sc.parts, sc.red, rt, Tw, wb, fg, a.ws, a.counters, epi);
      __syncthreads();
      tw += Tw;
    }
    sbase += T * nc;
  }
  return true;
}

// ------------------------------------------- tensor-parallel exchange

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Tensor parallel, after a phase whose epilogue stored its partial sums into
// every rank's exchange slot (kEpiTpPartial): this CTA's share of the row
// tiles of the sum, before the grid barrier that ends the phase. Row i:
//   y[i] = resid[i] + part_0[i] + ... + part_{n-1}[i]
// in rank order (the same on every rank, so every rank holds bit-identical
// residuals), each partial read until it carries this exchange step's tag
// (bounded), and the tile's sum of squares into ss_out with the residual
// epilogue's tree, from which the next RMSNorm takes its statistic. Every CTA
// of every rank reads only its own tiles' n words per row, all issued at
// once, so the next phase stages x like a single GPU. Returns false (block-
// uniform) when a read gave up. Out of line: its registers stay out of the
// GEMV loop's budget.
__device__ __noinline__ bool tp_reduce_slice(StepShared& sh, const StepGemv& g,
                                             const StepArgs& a) {
  const EpiParams& e = g.epi;
  const TpXchg* x = a.tp;
  const int n = x->n, dim = x->dim;
  const unsigned long long tag = sh.tp_gen0 + (unsigned int)g.tp_ar + 1u;
  const unsigned long long* parts =
      reinterpret_cast<const unsigned long long*>(x->peers[x->me] + x->parts_off) +
      (size_t)e.tp_slot * n * dim;
  const float* prev = e.resid ? e.resid : a.embedding + (size_t)sh.token * a.dim;
  const int ntile = (e.n_out + 15) / 16;
  const int lo = (int)((long long)ntile * blockIdx.x / gridDim.x);
  const int hi = (int)((long long)ntile * (blockIdx.x + 1) / gridDim.x);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long t0 = clock64();
  for (int t = lo + warp; t < hi; t += kStepWarps) {
    const int row = t * 16 + lane;
    const bool mine = lane < 16 && row < e.n_out;
    float v = 0.0f;
    if (mine) {
      unsigned long long w[kMaxTp];
#pragma unroll
      for (int r = 0; r < kMaxTp; ++r)
        if (r < n) w[r] = ld_relaxed_sys_u64(parts + (size_t)r * dim + row);
      v = __ldcg(prev + row);
#pragma unroll
      for (int r = 0; r < kMaxTp; ++r) {
        if (r >= n) break;
        while ((w[r] >> 32) != tag) {
          if (clock64() - t0 > kWaitCycles || *(volatile int*)&sh.tp_fail) {
            if (atomicCAS(&a.status->code, 0, MLB_ERR_TIMEOUT) == 0)
              atomicExch(&a.status->where, 400);
            *(volatile int*)&sh.tp_fail = 1;
            w[r] = tag << 32;
            break;
          }
          w[r] = ld_relaxed_sys_u64(parts + (size_t)r * dim + row);
        }
        v = __fadd_rn(v, __uint_as_float((unsigned int)w[r]));
      }
      e.y[row] = v;
    }
    float sq = mine ? v * v : 0.0f;
    sq += __shfl_xor_sync(0xffffffffu, sq, 8);
    sq += __shfl_xor_sync(0xffffffffu, sq, 4);
    sq += __shfl_xor_sync(0xffffffffu, sq, 2);
    sq += __shfl_xor_sync(0xffffffffu, sq, 1);
    if (lane == 0) e.ss_out[t] = sq;
  }
  __syncthreads();
  return !sh.tp_fail;
}

// ------------------------------------------------------ attention phase

// Sums NV values across the warp. On return v[0] of lane L holds the total of
// value index L / (32 / NV) (NV a power of two <= 32): each round keeps half of
// the remaining values and adds the partner lane's copy of that half.
template <int NV>
__device__ __forceinline__ void warp_multi_sum(float (&v)[NV], int lane) {
  static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "NV must be a power of two");
#pragma unroll
  for (int r = 0; r < 5; ++r) {
    const int off = 16 >> r;
    const int cnt = NV >> r;  // values still held (>= 1 once r >= log2 NV)
    if (cnt > 1) {
      const int half = cnt >> 1;
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? v[i] : v[i + half];
        const float keep = upper ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
}


struct AttnScratch {
  float* wpart;   // [warps][gq][attn_rec(D)]: m, l, -, -, o
  float* sc;      // [warps][NV] scores, then probabilities
  float* alpha;   // [warps][HG]
  float* ew;      // [gq][kMaxGrid] combine weights
  float* lw;      // [gq] combined l
};

template <int HG>
__device__ __forceinline__ AttnScratch attn_scratch(uint8_t* scratch, int D, int gq) {
  AttnScratch s;
  s.wpart = reinterpret_cast<float*>(scratch);
  s.sc = s.wpart + (size_t)kStepWarps * gq * attn_rec(D);
  s.alpha = s.sc + kStepWarps * AttnShape<HG>::NV;
  s.lw = s.alpha + kStepWarps * HG;
  s.ew = s.lw + gq;
  return s;
}

// Combines nrec records (m, l, o[D]) per query head into out[h][D] (o / l).
// rec(h, i) returns the record's base pointer; ld reads a float of it. Block-
// wide; ends synchronised.
template <class RecF>
__device__ __forceinline__ void attn_combine(const AttnScratch& s, int D, int gq, int nrec,
                                             RecF rec, bool from_global, float* out) {
  if ((int)threadIdx.x < gq) {
    const int h = threadIdx.x;
    float m = -INFINITY;
    for (int i = 0; i < nrec; ++i) {
      const float* r = rec(h, i);
      m = fmaxf(m, from_global ? __ldcg(r) : r[0]);
    }
    float l = 0.0f;
    for (int i = 0; i < nrec; ++i) {
      const float* r = rec(h, i);
      const float mi = from_global ? __ldcg(r) : r[0];
      const float li = from_global ? __ldcg(r + 1) : r[1];
      const float e = mi == -INFINITY ? 0.0f : expf(mi - m);
      s.ew[h * kMaxGrid + i] = e;
      l = fmaf(li, e, l);
    }
    s.lw[h] = l;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < gq * D; idx += kStepThreads) {
    const int h = idx / D, d = idx - h * D;
    float acc = 0.0f;
    for (int i = 0; i < nrec; ++i) {
      const float* r = rec(h, i) + kRecO + d;
      acc = fmaf(from_global ? __ldcg(r) : r[0], s.ew[h * kMaxGrid + i], acc);
    }
    out[(size_t)h * D + d] = __fdiv_rn(acc, s.lw[h]);
  }
  __syncthreads();
}

// Four K or V elements of a cache row through L2 (ld.global.cg) as loaded:
// fp32 a float4, bf16 a uint2 widened only when the block is used.
template <bool BF>
struct StepKv {
  using T = float4;
  static __device__ __forceinline__ T load(const uint8_t* p) {
    return __ldcg(reinterpret_cast<const float4*>(p));
  }
  static __device__ __forceinline__ T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  static __device__ __forceinline__ float4 widen(const T& v) { return v; }
};
template <>
struct StepKv<true> {
  using T = uint2;
  static __device__ __forceinline__ T load(const uint8_t* p) {
    return __ldcg(reinterpret_cast<const uint2*>(p));
  }
  static __device__ __forceinline__ T zero() { return make_uint2(0u, 0u); }
  static __device__ __forceinline__ float4 widen(const T& u) { return KvRaw<true>::widen(u); }
};

// One warp: positions [t0, t1) of a piece of KV head kvh, blocks of PB
// positions round robin over warps; online softmax per query head. Query
// heads go HG at a time (each pass re-reads the block's K/V rows, from L2).
// BF: the cache holds bf16 elements.
template <int HG, bool BF>
__device__ __forceinline__ void attn_warp(const StepAttn& at, const AttnScratch& s, int gq,
                                          int kvh, int t0, int t1, int v_end, int warp,
                                          int lane) {
  constexpr int PB = AttnShape<HG>::PB, NV = AttnShape<HG>::NV;
  constexpr unsigned kNvMask = (1u << NV) - 1u;  // lanes < NV
  const int D = at.D, nvec = D >> 2, rec = attn_rec(D);
  const bool dl = lane < nvec;
  using Kv = StepKv<BF>;
  using KvT = typename Kv::T;
  constexpr size_t esz = BF ? 2 : 4;
  const size_t row = (size_t)at.KV * D * esz;  // bytes from one position to the next
  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(at.keys) + ((size_t)kvh * D + 4 * lane) * esz;
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(at.values) + ((size_t)kvh * D + 4 * lane) * esz;
  float* scw = s.sc + warp * NV;
  float* alw = s.alpha + warp * HG;
  float* wp = s.wpart + (size_t)warp * gq * rec;
#pragma unroll 1
  for (int hg = 0; hg < gq; hg += HG) {
    float4 q[HG], o[HG];
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      q[h] = (dl && hg + h < gq)
                 ? __ldcg(reinterpret_cast<const float4*>(at.q + (size_t)(kvh * gq + hg + h) * D) +
                          lane)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
      o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // lane i < NV keeps (m, l) of query head hg + i / PB
    float m_run = -INFINITY, l_run = 0.0f;
    // K and V rows of block tb (zero past the slice)
    auto load_block = [&](int tb, KvT (&kx)[PB], KvT (&vx)[PB]) {
#pragma unroll
      for (int j = 0; j < PB; ++j) {
        const int t = tb + j;
        kx[j] = (dl && t < t1) ? Kv::load(kbase + (size_t)t * row) : Kv::zero();
        vx[j] = (dl && t < t1 && t < v_end) ? Kv::load(vbase + (size_t)t * row) : Kv::zero();
      }
    };
    // narrow passes keep the next block's rows in flight while this one is
    // computed (wider passes have no registers to spare)
    constexpr bool kPipe = HG <= 2;
    KvT kn[PB], vn[PB];
    if (kPipe) load_block(t0 + warp * PB, kn, vn);
    for (int tb = t0 + warp * PB; tb < t1; tb += kStepWarps * PB) {
      float4 kx[PB], vx[PB];
      if (kPipe) {
#pragma unroll
        for (int j = 0; j < PB; ++j) {
          kx[j] = Kv::widen(kn[j]);
          vx[j] = Kv::widen(vn[j]);
        }
        if (tb + kStepWarps * PB < t1) load_block(tb + kStepWarps * PB, kn, vn);
      } else {
        KvT kr[PB], vr[PB];
        load_block(tb, kr, vr);
#pragma unroll
        for (int j = 0; j < PB; ++j) {
          kx[j] = Kv::widen(kr[j]);
          vx[j] = Kv::widen(vr[j]);
        }
      }
      float dv[NV];
#pragma unroll
      for (int h = 0; h < HG; ++h)
#pragma unroll
        for (int j = 0; j < PB; ++j) {
          float d = q[h].x * kx[j].x;
          d = fmaf(q[h].y, kx[j].y, d);
          d = fmaf(q[h].z, kx[j].z, d);
          d = fmaf(q[h].w, kx[j].w, d);
          dv[h * PB + j] = d;
        }
      warp_multi_sum<NV>(dv, lane);
      if ((lane & (32 / NV - 1)) == 0) scw[lane / (32 / NV)] = dv[0];
      __syncwarp();
      if (lane < NV) {
        const int j = lane % PB;
        const int t = tb + j;
        const float sc = t < t1 ? __fmul_rn(scw[lane], at.scale) : -INFINITY;
        float bmax = sc;
#pragma unroll
        for (int off = 1; off < PB; off <<= 1)
          bmax = fmaxf(bmax, __shfl_xor_sync(kNvMask, bmax, off));
        const float mnew = fmaxf(m_run, bmax);
        const float p = t < t1 ? expf(sc - mnew) : 0.0f;
        float psum = p;
#pragma unroll
        for (int off = 1; off < PB; off <<= 1) psum += __shfl_xor_sync(kNvMask, psum, off);
        const float al = m_run == -INFINITY ? 0.0f : expf(m_run - mnew);
        l_run = fmaf(l_run, al, psum);
        m_run = mnew;
        scw[lane] = t < v_end ? p : 0.0f;  // softmax weight counted, V row summed below v_end
        if (j == 0) alw[lane / PB] = al;
      }
      __syncwarp();
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        const float al = alw[h];
        float4 acc = make_float4(o[h].x * al, o[h].y * al, o[h].z * al, o[h].w * al);
#pragma unroll
        for (int j = 0; j < PB; ++j) {
          const float p = scw[h * PB + j];
          acc.x = fmaf(p, vx[j].x, acc.x);
          acc.y = fmaf(p, vx[j].y, acc.y);
          acc.z = fmaf(p, vx[j].z, acc.z);
          acc.w = fmaf(p, vx[j].w, acc.w);
        }
        o[h] = acc;
      }
      __syncwarp();
    }
    // this warp's record per query head of the pass
    if (lane < NV && lane % PB == 0 && hg + lane / PB < gq) {
      wp[(hg + lane / PB) * rec] = m_run;
      wp[(hg + lane / PB) * rec + 1] = l_run;
    }
    if (dl) {
#pragma unroll
      for (int h = 0; h < HG; ++h)
        if (hg + h < gq)
          *reinterpret_cast<float4*>(wp + (hg + h) * rec + kRecO + 4 * lane) = o[h];
    }
  }
}

template <int HG>
__device__ __noinline__ bool attn_phase(StepShared& sh, const StepPhase& cur, uint8_t* scratch,
                           const StepArgs& a) {
  const StepAttn& at = cur.at;
  const int D = at.D, rec = attn_rec(D);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = sh.pos;
  const int n = pos + 1;
  const int v_end = at.include_current_v ? (int)n : pos;
  const int G = gridDim.x;
  const int gq = at.H / at.KV;
  const AttnScratch s = attn_scratch<HG>(scratch, D, gq);
  // Work items: each KV head cut into pph equal position slices, one item per
  // CTA (CTAs past the items idle), so no CTA carries two pieces.
  const int pph = max(1, min(G / at.KV, n));
  const int items = at.KV * pph;
  for (int item = blockIdx.x; item < items; item += G) {
    const int kvh = item / pph, piece = item - kvh * pph;
    const int t0 = n * piece / pph, t1 = n * (piece + 1) / pph;
    if (at.kv_bf16)
      attn_warp<HG, true>(at, s, gq, kvh, t0, t1, v_end, warp, lane);
    else
      attn_warp<HG, false>(at, s, gq, kvh, t0, t1, v_end, warp, lane);
    __syncthreads();
    float* out = at.out + (size_t)kvh * gq * D;
    if (pph == 1) {
      attn_combine(s, D, gq, kStepWarps,
                   [&](int h, int i) { return s.wpart + ((size_t)i * gq + h) * rec; }, false, out);
      continue;
    }
    // this piece's record: the warps combined, unnormalised (m, l, o)
    float* dst = a.attn_ws + (size_t)item * gq * rec;
    if (warp < gq) {  // warp h combines the 16 warp records of query head h
      const int h = warp;
      const bool has = lane < kStepWarps;
      const float* r = s.wpart + ((size_t)(has ? lane : 0) * gq + h) * rec;
      const float mi = has ? r[0] : -INFINITY;
      float m = mi;
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      const float e = (has && mi != -INFINITY) ? expf(mi - m) : 0.0f;
      float l = has ? r[1] * e : 0.0f;
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (has) s.ew[h * kMaxGrid + lane] = e;
      if (lane == 0) {
        dst[h * rec] = m;
        dst[h * rec + 1] = l;
      }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < gq * D; idx += kStepThreads) {
      const int h = idx / D, d = idx - h * D;
      float acc = 0.0f;
      for (int i = 0; i < kStepWarps; ++i)
        acc = fmaf(s.wpart[((size_t)i * gq + h) * rec + kRecO + d], s.ew[h * kMaxGrid + i], acc);
      dst[h * rec + kRecO + d] = acc;
    }
    // thread 0 publishes the CTA's record and, as the head's last slice,
    // acquires the others' before the block reads them: one acq_rel add
    // after bar.sync (the pattern of a grid barrier)
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned int prev;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                   : "=r"(prev)
                   : "l"(a.attn_counters + kvh)
                   : "memory");
      sh.flag = (int)prev == pph - 1;
    }
    __syncthreads();
    if (sh.flag) {
      // The last slice of the head to finish combines all slices, in order:
      // their records are copied into the scratch past the attention's own
      // (one round trip for all of them) when they fit, else read in place.
      const float* src = a.attn_ws + (size_t)kvh * pph * gq * rec;
      const size_t own = ((size_t)((s.ew + gq * kMaxGrid) - reinterpret_cast<float*>(scratch)) *
                              4 + 127) / 128 * 128;
      const size_t need = (size_t)pph * gq * rec * 4;
      if (own + need <= (size_t)a.scratch_bytes) {
        float* rs = reinterpret_cast<float*>(scratch + own);
        for (int i = threadIdx.x; i < (int)(need / 16); i += kStepThreads)
          cp_async16(reinterpret_cast<float4*>(rs) + i, reinterpret_cast<const float4*>(src) + i);
        cp_async_commit();
        cp_async_wait_all();
        __syncthreads();
        attn_combine(s, D, gq, pph,
                     [&](int h, int i) { return rs + ((size_t)i * gq + h) * rec; }, false, out);
      } else {
        attn_combine(s, D, gq, pph,
                     [&](int h, int i) { return src + ((size_t)i * gq + h) * rec; }, true, out);
      }
      if (threadIdx.x == 0) a.attn_counters[kvh] = 0;
    }
    __syncthreads();
  }
  return true;
}

// ---------------------------------------------------------------- kernel

template <int QT, int HG>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepArgs args) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring_base = smem;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem + (size_t)kStepWarps * args.stages * args.sb_stride);
  uint8_t* scratch = reinterpret_cast<uint8_t*>(bars + kStepWarps * kMaxStages);
  StepShared& sh = *reinterpret_cast<StepShared*>(scratch + args.scratch_bytes);
  if (threadIdx.x == 0) sh.args = args;
  __syncthreads();
  const StepArgs& a = sh.args;
  StepCta* tab = reinterpret_cast<StepCta*>(reinterpret_cast<uint8_t*>(&sh) +
                                            (sizeof(StepShared) + 15) / 16 * 16);
  // this CTA's column of the phase table
  constexpr int kCta16 = (int)(sizeof(StepCta) / 16);
  for (int i = threadIdx.x; i < kCta16 * a.nphases; i += kStepThreads)
    reinterpret_cast<int4*>(tab)[i] = __ldg(
        reinterpret_cast<const int4*>(a.cta + (size_t)(i / kCta16) * gridDim.x + blockIdx.x) +
        i % kCta16);
  // an earlier step failed: do nothing (one read, shared by the block)
  if (threadIdx.x == 0) {
    sh.pos = *a.pos;
    sh.token = *a.token;
    sh.flag = *(volatile int*)&a.status->code;
    sh.tp_gen0 = a.tp ? *(volatile unsigned int*)a.tp_gen : 0u;
    sh.tp_fail = 0;
    sh.tp_kgen0 = a.tp ? *(volatile unsigned int*)(a.tp_gen + 1) : 0u;
  }
  __syncthreads();
  if (sh.flag != 0) return;
  __syncthreads();

  Ring rg;
  rg.base = ring_base + (size_t)warp * a.stages * a.sb_stride;
  rg.bars = bars + warp * kMaxStages;
  rg.stride = a.sb_stride;
  rg.stages = a.stages;
  rg.slot = 0;
  rg.parity = 0;
  rg.inflight = 0;
  Producer& pr = sh.prod[warp];
  ProducerRun run{nullptr, 0, 0};
  if (lane == 0) pr.p = 0;
  if (lane == 0) {
    for (int s = 0; s < a.stages; ++s) mbar_init(&rg.bars[s], 1);
    fence_mbar_init();
    fence_proxy_async_smem();
    producer_seek(pr, tab, a.nphases, warp);
    run = producer_load_run(pr, tab, a.nphases, a.sb_stride);
    for (int s = 0; s < a.stages; ++s)
      producer_issue(pr, run, rg, s, tab, a.nphases, warp, a.sb_stride);
  }
  __syncwarp();

  // Phase descriptors: the first one now, each later one prefetched with
  // cp.async while the phase before it runs (complete and visible after that
  // phase's grid barrier).
  constexpr int kDesc16 = (int)(sizeof(StepPhase) / 16);
  for (int i = threadIdx.x; i < kDesc16; i += kStepThreads)
    reinterpret_cast<int4*>(&sh.cur[0])[i] = __ldg(reinterpret_cast<const int4*>(a.phases) + i);
  bool ok = true;
  unsigned int nbar = 0;  // grid barriers passed
  for (int p = 0; p < a.nphases && ok; ++p) {
    StepPhase& cur = sh.cur[p & 1];
    if (threadIdx.x == 0) sh.flag = 1;
    __syncthreads();
    if (a.trace && threadIdx.x == 0)
      a.trace[((size_t)p * gridDim.x + blockIdx.x) * 2] = global_ns();
    if (p + 1 < a.nphases) {
      const int4* src = reinterpret_cast<const int4*>(a.phases + p + 1);
      int4* dst = reinterpret_cast<int4*>(&sh.cur[(p + 1) & 1]);
      for (int i = threadIdx.x; i < kDesc16; i += kStepThreads) cp_async16(dst + i, src + i);
      cp_async_commit();
    }
    if (cur.kind == kPhaseGemv) {
      ok = gemv_phase<QT>(sh, cur, tab[p], scratch, rg, pr, run, tab, a);
      // tensor parallel: this phase's partial sums, added across ranks
      if (ok && cur.g.tp_ar >= 0) ok = tp_reduce_slice(sh, cur.g, a);
    } else {
      ok = attn_phase<HG>(sh, cur, scratch, a);
    }
    cp_async_wait_all();
    if (a.trace && threadIdx.x == 0)
      a.trace[((size_t)p * gridDim.x + blockIdx.x) * 2 + 1] = global_ns();
    if (ok && p + 1 < a.nphases)
      ok = grid_barrier(&a.sync[0], ++nbar, a.status, 100 + p, &sh.flag);
  }
  if (!ok) {
    if (lane == 0) ring_drain(rg.bars, rg.stages, rg.slot, rg.parity, rg.inflight);
    return;
  }
  // End of step: the last CTA to finish publishes the greedy token and
  // advances the position (step_finalize_kernel's job on the per-op path).
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.sync[1], 1u) == gridDim.x - 1) {
      __threadfence();
      unsigned long long key = atomicOr(a.argmax_key, 0ull);
      if (a.tp) {
        // the greedy token across vocabulary shards: every rank's key into
        // every buffer, the last exchange step of the decode step, then the
        // same maximum on every rank
        const TpXchg* x = a.tp;
        for (int r = 0; r < x->n; ++r)
          reinterpret_cast<unsigned long long*>(x->peers[r] + x->keys_off)[x->me] = key;
        __threadfence_system();
        for (int r = 0; r < x->n; ++r)
          red_release_sys_add(reinterpret_cast<unsigned int*>(x->peers[r] + x->kflags_off) + x->me,
                              1u);
        const unsigned int kdone = sh.tp_kgen0 + 1u;
        if (tp_wait_all(x, x->kflags_off, kdone, true, a.status, 299)) {
          const unsigned long long* keys =
              reinterpret_cast<const unsigned long long*>(x->peers[x->me] + x->keys_off);
          for (int r = 0; r < x->n; ++r) {
            const unsigned long long kr = __ldcg(keys + r);
            key = kr > key ? kr : key;
          }
        }
        a.tp_gen[0] = sh.tp_gen0 + (unsigned int)a.tp_steps;
        a.tp_gen[1] = kdone;
      }
      const int t = argmax_index_of(key);
      *a.token = t;
      a.tokens[*a.step] = t;
      *a.step += 1;
      *a.pos += 1;
      *a.argmax_key = 0ull;
      a.sync[0] = 0u;
      a.sync[1] = 0u;
      __threadfence();
    }
  }
}

// Pass width for a GQA group size: 1 and 2 exactly, 4 for every larger group.
int pass_heads(int gq) { return gq <= 2 ? gq : 4; }

template <int QT>
void* pick_kernel(int hg) {
  switch (hg) {
    case 1: return (void*)decode_step_kernel<QT, 1>;
    case 2: return (void*)decode_step_kernel<QT, 2>;
    default: return (void*)decode_step_kernel<QT, 4>;
  }
}

void* step_kernel_ptr(int qtype, int gq) {
  const int hg = pass_heads(gq);
  if (qtype == MLB_Q4_0) return pick_kernel<MLB_Q4_0>(hg);
  if (qtype == MLB_Q4_1) return pick_kernel<MLB_Q4_1>(hg);
  return pick_kernel<MLB_Q8_0>(hg);
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

namespace {

// The step kernel's two waits, each made to wait for something that never
// comes: which = 0 an mbarrier phase that nothing completes (a ring slot whose
// copy never lands), which = 1 a grid barrier that the launch's only CTA can
// never fill (a CTA that never arrives). Each gives up after `limit` cycles
// and records MLB_ERR_TIMEOUT at `where` in *st.
__global__ void wait_selftest_kernel(DeviceStatus* st, unsigned int* counter, int which,
                                     long long limit, int where) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int flag;
  if (which == 0) {
    if (threadIdx.x == 0) {
      mbar_init(&bar, 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !mbar_try_wait(&bar, 0)) mbar_wait_bounded(&bar, 0, st, where, limit);
  } else {
    grid_barrier(counter, 2, st, where, &flag, limit);
  }
}

}  // namespace

void step_wait_selftest(int which, long long limit_cycles, int where, int* code, int* at) {
  DeviceStatus* st = nullptr;
  unsigned int* counter = nullptr;
  MLB_CUDA(cudaMalloc(&st, sizeof(DeviceStatus)));
  cudaError_t e = cudaMalloc(&counter, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(st, 0, sizeof(DeviceStatus));
  if (e == cudaSuccess) e = cudaMemset(counter, 0, sizeof(unsigned int));
  if (e == cudaSuccess) {
    wait_selftest_kernel<<<1, 32>>>(st, counter, which, limit_cycles, where);
    e = cudaGetLastError();
  }
  DeviceStatus h{};
  if (e == cudaSuccess) e = cudaMemcpy(&h, st, sizeof(h), cudaMemcpyDeviceToHost);
  cudaFree(counter);
  cudaFree(st);
  MLB_CUDA(e);
  *code = h.code;
  *at = h.where;
}

size_t step_smem_bytes(int scratch_bytes, int sb_stride, int stages, int nphases) {
  return (size_t)kStepWarps * stages * sb_stride + (size_t)kStepWarps * kMaxStages * 8 +
         (size_t)scratch_bytes + round_up(sizeof(StepShared), 16) +
         (size_t)nphases * sizeof(StepCta);
}

std::vector<StepCta> step_cta_table(const std::vector<StepPhase>& ph, int grid) {
  const int nph = (int)ph.size();
  std::vector<StepCta> t((size_t)nph * grid);
  int next = nph;  // the first GEMV phase after the current one, walking backwards
  for (int i = nph - 1; i >= 0; --i) {
    for (int c = 0; c < grid; ++c) {
      StepCta& e = t[(size_t)i * grid + c];
      e = StepCta{};
      e.next = next;
      if (ph[i].kind != kPhaseGemv) continue;
      const StepGemv& g = ph[i].g;
      e.cb = cta_start(c, grid, g.ntiles, g.nchunks, g.gc, g.ngroups);
      e.ce = cta_start(c + 1, grid, g.ntiles, g.nchunks, g.gc, g.ngroups);
      e.w = g.w + (size_t)e.cb * g.sbb;
      // segments: the range's group-tiles of each chunk group
      for (int u = e.cb; u < e.ce;) {
        if (e.nseg == 2) fail(MLB_ERR_INVALID, "decode step kernel: range over three chunk groups");
        const SbPos sp = sb_decode(u, g.ntiles, g.nchunks, g.gc);
        const int group_end = (sp.grp + 1) * g.ntiles * g.gc;  // past the group's super-blocks
        const int end = std::min(e.ce, std::min(group_end, g.ntiles * g.nchunks));
        e.T[e.nseg] = (end - u) / sp.geff;
        e.nc[e.nseg] = sp.geff;
        e.grp[e.nseg] = sp.grp;
        e.t0[e.nseg] = sp.t;
        ++e.nseg;
        u = end;
      }
    }
    if (ph[i].kind == kPhaseGemv) next = i;
  }
  return t;
}

int step_gemv_scratch(const QMatrix& m) {
  const int nslots = m.ngroups > 1 ? 2 : 1;
  size_t b = (size_t)nslots * m.gc * frag_chunk_u32<1>() * 4;
  b += (size_t)nslots * m.gc * 8 * 4 * (m.qtype == MLB_Q4_1 ? 2 : 1);  // side data
  b += (size_t)win_sbs<1>() * 16 * 4;  // super-block partials
  b += (size_t)kStepWarps * (16 + kSegList) * 4;
  return (int)round_up(b, 128);
}

int step_attn_scratch(int gq, int D) {
  const int hg = pass_heads(gq), nv = hg * 4;
  size_t b = (size_t)kStepWarps * gq * attn_rec(D) * 4 + (size_t)kStepWarps * nv * 4 +
             (size_t)kStepWarps * hg * 4 + (size_t)gq * 4 + (size_t)gq * kMaxGrid * 4;
  return (int)round_up(b, 128);
}

bool step_gemv_ok(const QMatrix& m, int grid, std::string* why) {
  if (m.qtype != MLB_Q4_0 && m.qtype != MLB_Q4_1 && m.qtype != MLB_Q8_0) {
    *why = "a projection is not Q4_0/Q4_1/Q8_0";
    return false;
  }
  // at most two chunk groups per CTA range (the staged activations)
  for (long long c = 0; c < grid; ++c) {
    const int cb = cta_start((int)c, grid, m.ntiles, m.nchunks, m.gc, m.ngroups);
    const int ce = cta_start((int)c + 1, grid, m.ntiles, m.nchunks, m.gc, m.ngroups);
    if (cb >= ce) continue;
    const int g0 = sb_decode(cb, m.ntiles, m.nchunks, m.gc).grp;
    const int g1 = sb_decode(ce - 1, m.ntiles, m.nchunks, m.gc).grp;
    if (g1 - g0 > 1) {
      *why = "a CTA range spans more than two chunk groups";
      return false;
    }
  }
  return true;
}

bool step_attn_ok(int H, int KV, int D, std::string* why) {
  const int gq = H / KV;
  if (D % 4 != 0 || D > 128) {
    *why = "head_dim must be a multiple of 4 and at most 128";
    return false;
  }
  if (step_attn_scratch(gq, D) > 160 * 1024) {
    *why = "the GQA group is too large for the attention scratch";
    return false;
  }
  return true;
}

void step_launch(const StepPlan& plan, const StepArgs& args, cudaStream_t stream) {
  if (!plan.ok) invalid("decode step kernel: " + plan.why);
  if (plan.grid > kMaxGrid) invalid("decode step kernel: grid too large");
  void* fn = step_kernel_ptr(plan.qtype, plan.gq);
  int dev = 0;
  MLB_CUDA(cudaGetDevice(&dev));
  static size_t smem_set[64][3][3] = {};
  const int qi = plan.qtype == MLB_Q4_0 ? 0 : (plan.qtype == MLB_Q4_1 ? 1 : 2);
  const int gi = pass_heads(plan.gq) == 1 ? 0 : (pass_heads(plan.gq) == 2 ? 1 : 2);
  if (dev < 64 && smem_set[dev][qi][gi] < plan.smem) {
    MLB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)plan.smem));
    smem_set[dev][qi][gi] = plan.smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)plan.grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<StepArgs*>(&args)};
  MLB_CUDA(cudaLaunchKernelExC(&cfg, fn, params));
}

// Checks done once per context: the step kernel's block fits one per SM.
int step_max_blocks_per_sm(int qtype, int gq, size_t smem) {
  void* fn = step_kernel_ptr(qtype, gq);
  MLB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int n = 0;
  MLB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kStepThreads, smem));
  return n;
}

}  // namespace mlb
