// The whole top-k MoE layer for a decode-sized batch in one launch.
//
// Included by moe_gemm.cu (same translation unit: device error flag, kernel
// clocks, tensor maps, PTX wrappers). For at most kDecodeMaxTokens tokens
// (the MMA's N = 16) and kDecodeMaxSlots routed slots, the layer's stages —
// routing align, gate_up GEMM + SwiGLU, down GEMM + weighted combine, output
// conversion — run as phases of one persistent kernel, one CTA per SM:
//
//   phase 0  every CTA reads the top-k ids and weights (at most 128 slots)
//            — or, given the router logits, routes the tokens itself, one
//            warp per token (route.cuh; CTA 0 writes the ids and weights
//            out) — and derives the active experts (distinct valid ids in increasing
//            order; expert tile m = the m-th of them) and, per (tile, token),
//            the token's summed routing weight for that expert; its share of
//            the fp32 output accumulator, the group counts and the readiness
//            counts is cleared, then the CTA arrives on the launch counter
//            (nothing waits there)
//   phase 1  gate_up work items (tile m, 128-feature tile f, K split s):
//            weights as the MMA's 128-row operand (gate and up rows, two
//            accumulators), the N = 16 operand is x itself — the first 16 rows
//            of x, rows past T zero-filled by TMA — so there is no gather.
//            SwiGLU output h[m][t][i] for all T tokens of the tile (tokens not
//            routed to the expert are computed and never used); with K split,
//            each split stores fp32 partial sums and the last split of a unit
//            to finish (a count per epilogue warp) adds them in split order and
//            applies SwiGLU. Each warp that stores its 32 features of tile m
//            adds one to tile m's readiness count (one atomic: its waiters
//            and adders first check that every CTA has arrived on the launch
//            counter, long true by then, so the count was cleared)
//   phase 2  down work items (tile m, 128-output-feature tile): the producer
//            loads the item's weights at once and h[m] (16 rows) once tile m's
//            readiness count is full — no device-wide barrier, so the down
//            phase of one expert overlaps the gate_up phase of others; the
//            epilogue, once every CTA has arrived on the launch counter (its
//            clears are done), adds weight(m, t) * acc into the fp32
//            accumulator row of token t, then counts the add per (token,
//            32-feature group); the warp whose add completes a group (its
//            token's distinct experts all added) converts it to the output
//            dtype
//
// The producer starts loading its first phase-2 weight tiles as soon as ring
// stages free up after its last phase-1 stage (the weights do not depend on
// h); only the h rows wait. At one token a phase-2 item's weights (128 rows x
// I) fit in the ring, so the down projection's weight stream overlaps the
// gate_up phase's tail.
//
// Cross-CTA state: a count and a generation word in static device memory
// (the launch counter: the last CTA to arrive clears the count and advances
// the generation, which every CTA read before arriving — the tag of this
// launch), tagged count words in the workspace for the K splits (a word
// left by an earlier launch carries another tag and counts as zero, so
// nothing clears them) and the cleared readiness counts. All CTAs are resident at once (grid <= SM
// count, one CTA per SM by its shared memory), and no CTA's phase-1 work
// waits on another CTA. Every wait is bounded; a cross-CTA wait that times
// out latches device error 7, and moe_get_device_error() resets the launch
// counter after any error. Two such launches must not overlap on one GPU
// (different streams).
#include <type_traits>

#include "route.cuh"

namespace moe {
namespace {

constexpr int kDecodeMaxTokens = 16;
constexpr int kDecodeMaxSlots = 128;
constexpr int kDecodeRouteMaxExperts = 256;  // routing in phase 0: 8 logits per lane
constexpr int kDecodeMaxSplits = 8;  // K splits of the gate_up phase
constexpr int DK_STAGE_A = 2 * SW_A_TILE;                  // 32 KB: gate + up tiles, or two w2 K blocks
constexpr int DK_STAGE_B = 2 * kDecodeMaxTokens * ROW_BYTES;  // 4 KB: token boxes for the A tiles
constexpr int DK_STAGE = DK_STAGE_A + DK_STAGE_B;
constexpr int DK_STAGES = 6;
constexpr int DK_TMEM_COLS = 64;                           // 2 buffers x (gate 16 + up 16) columns
// cluster K-split reduction: the leader CTA's buffer for the other splits'
// gate and up sums, [split - 1][128 features][2][T] floats
constexpr int kDecodeRedBytes = 6144;

__device__ unsigned int g_decode_bar_count = 0;
__device__ unsigned int g_decode_bar_gen = 0;

// Launch counter (one thread per CTA, after the CTA's phase-0 clears):
// the last CTA to arrive resets the count and advances the generation, so
// the generation a CTA reads before arriving is the same for every CTA of
// the launch and differs from launch to launch. Nothing waits here.
__device__ void decode_launch_arrive(unsigned int nblocks) {
  __threadfence();
  if (atomicAdd(&g_decode_bar_count, 1u) == nblocks - 1u) {
    atomicExch(&g_decode_bar_count, 0u);
    __threadfence();
    atomicAdd(&g_decode_bar_gen, 1u);
  }
}

// Waits until every CTA of the launch has arrived (the generation moved on
// from `gen`). Returns false after the time limit or when *abort is raised.
__device__ bool decode_all_arrived(unsigned int gen, volatile int* abort) {
  volatile unsigned int* gen_p = &g_decode_bar_gen;
  const uint64_t t0 = ptx::globaltimer();
  while (*gen_p == gen) {
    if (*abort) return false;
    if (ptx::globaltimer() - t0 > MOE_WAIT_TIMEOUT_NS) return false;
    __nanosleep(64);
  }
  __threadfence();
  return true;
}

// Counts one arrival on a 64-bit counter word in caller memory that nothing
// clears: bits [16, 64) hold the launch's tag, [0, 16) the count. A word
// whose tag differs (left by an earlier launch, or never written) counts as
// zero. Returns 1 for the arrival that makes the count `total`, 0 otherwise,
// -1 if the word stayed contended past a bound.
__device__ __forceinline__ int tagged_count_last(unsigned long long* ctr, unsigned long long tag,
                                                 unsigned int total) {
  unsigned long long old = atomicAdd(ctr, 0ull);
  for (int tries = 0; tries < 256; ++tries) {
    const unsigned int cnt = ((old >> 16) == (tag >> 16)) ? (unsigned int)(old & 0xFFFFull) : 0u;
    const unsigned long long prev = atomicCAS(ctr, old, (tag & ~0xFFFFull) | (cnt + 1));
    if (prev == old) return cnt + 1 == total ? 1 : 0;
    old = prev;
  }
  return -1;
}

// Waits until a count word holds at least `total`. Returns false after the
// time limit or when *abort is raised.
__device__ bool wait_count(const unsigned int* ctr, unsigned int total, volatile int* abort) {
  const volatile unsigned int* v = ctr;
  const uint64_t t0 = ptx::globaltimer();
  while (*v < total) {
    if (*abort) return false;
    if (ptx::globaltimer() - t0 > MOE_WAIT_TIMEOUT_NS) return false;
    __nanosleep(32);
  }
  __threadfence();
  return true;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// The gate_up phase's work: units u = m * nf1 + f (expert tile m, feature
// tile f) of kb1 K blocks each, spread over the G CTAs in one of two ways:
//   split  (sp >= 1, while units * sp <= G): CTA b < units * sp takes K split
//          b % sp of unit b / sp (balanced, non-empty ranges); sp = 1 is one
//          unit per CTA
//   waves  (sp = 0, more units than CTAs): whole units, CTA b taking units b,
//          b + G, ..., so each wave's expert tiles finish together and their
//          down phase starts while the next wave runs. (Splitting the
//          partial last wave along K over all CTAs measured slower: the
//          reduction of its partials costs more than the imbalance it
//          removes, which the down phase mostly overlaps anyway.)
// A unit split over several CTAs is a sum of fp32 partials, one slot per
// CTA.
struct P1Plan {
  int sp, kb1, units, G;
  // sp_fixed > 0: that split count (the cluster size of a cluster launch,
  // where each cluster holds one unit's splits)
  __device__ P1Plan(int units_, int kb1_, int G_, int sp_fixed) : kb1(kb1_), units(units_), G(G_) {
    if (sp_fixed > 0) sp = sp_fixed;
    else if (2 * units <= G && units > 0) sp = max(1, min(min(G / units, kDecodeMaxSplits), kb1 / 4));
    else sp = units <= G ? 1 : 0;
  }
  // segments (unit, K blocks [k0, k1)) of CTA b, in order
  struct Iter {
    const P1Plan& pl;
    int b, next_u;
    __device__ Iter(const P1Plan& p, int b_) : pl(p), b(b_), next_u(b_) {}
    __device__ bool next(int& u, int& k0, int& k1) {
      if (pl.sp) {
        if (next_u != b || b >= pl.units * pl.sp) return false;
        u = b / pl.sp;
        const int s = b % pl.sp;
        k0 = s * pl.kb1 / pl.sp;
        k1 = (s + 1) * pl.kb1 / pl.sp;
        next_u = -1;
        return true;
      }
      if (next_u >= pl.units) return false;
      u = next_u;
      k0 = 0;
      k1 = pl.kb1;
      next_u += pl.G;
      return true;
    }
  };
  // CTAs that compute unit u: [first, last], in K order
  __device__ void ctas(int u, int& first, int& last) const {
    if (sp) {
      first = u * sp;
      last = first + sp - 1;
    } else {
      first = last = u % G;
    }
  }
  // partial-sum slot of unit u's segment on CTA b (units split over CTAs only)
  __device__ int slot(int u, int b) const { return b; }
};

struct DecodeParams {
  int T, k, E, I, H;
  int nf1, nf2;          // feature tiles of 128: ceil(I / 128), ceil(H / 128)
  int kb1, kb2;          // K blocks of 128 bytes: gate_up (H), down (I)
  int max_tiles;         // tiles reserved in h: min(E, T * k)
  uint32_t idesc;        // M = 128, N = 16
  const int32_t* ids;    // [T, k]
  const float* wts;      // [T, k]
  void* h;               // [max_tiles][16][I], x dtype
  float* partial;        // [grid][2][128][16] partial sums of units split over several CTAs
  unsigned long long* split_cnt;  // [max_tiles * nf1][4] tagged counts (never cleared)
  unsigned int* h_ready;          // [max_tiles] finished (feature tile, warp) groups of h, cleared in phase 0
  float* y32;            // [T, H]
  int32_t* conv_cnt;     // [T][nf2 * 4] adds per (token, 32-feature group)
  void* y;               // [T, H], x dtype
  int dtype;             // MOE_BF16 or MOE_F16
  int clock_slot;
  int cluster_sp;        // > 0: launched as clusters of this many CTAs, each one gate_up unit's K splits,
                         // reduced through the leader's shared memory
  // routing in phase 0 (logits != nullptr; ids / wts unused): CTA 0
  // writes the routing to ids_out / wts_out
  const void* logits;    // [T, E] router logits
  int logits_dtype;      // MOE_F32, MOE_BF16 or MOE_F16
  int sigmoid, renormalize;
  int32_t* ids_out;      // [T, k]
  float* wts_out;        // [T, k]
};

template <int KIND>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    moe_decode_kernel(const __grid_constant__ CUtensorMap tmap_w13, const __grid_constant__ CUtensorMap tmap_w2,
                      const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_h,
                      const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + DK_STAGES * DK_STAGE);
  uint64_t* empty = full + DK_STAGES;
  uint64_t* tfull = empty + DK_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  unsigned int* s_gen = reinterpret_cast<unsigned int*>(tmem_slot + 3);  // launch generation
  // routing tables (phase 0)
  int32_t* s_act = reinterpret_cast<int32_t*>(smem + DK_STAGES * DK_STAGE + 256);  // [128] expert of tile m
  int32_t* s_ids = s_act + kDecodeMaxSlots;                                          // [128] slot ids
  float* s_w = reinterpret_cast<float*>(s_ids + kDecodeMaxSlots);                    // [128] slot weights
  int* s_key = reinterpret_cast<int*>(s_w + kDecodeMaxSlots);                        // [128] expert id of a first slot
  int* s_kd = s_key + kDecodeMaxSlots;                                             // [16] distinct experts per token
  float* s_red = reinterpret_cast<float*>(s_kd + 16);                                // cluster reduction buffer
  uint64_t* red_bar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(s_red) + kDecodeRedBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.T * p.k;
  constexpr int kElems = ROW_BYTES / (KIND == 0 ? 2 : 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < DK_STAGES; ++i) {
      ptx::mbar_init(&full[i], 1);
      ptx::mbar_init(&empty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      ptx::mbar_init(&tempty[a], 4 * 32);
    }
    ptx::mbar_init(drain, 1);
    // cluster launch: one arrival per epilogue warp of every other split
    if (p.cluster_sp > 0) ptx::mbar_init(red_bar, 4 * (p.cluster_sp - 1));
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_w13);
    ptx::prefetch_tmap(&tmap_w2);
    ptx::prefetch_tmap(&tmap_x);
    ptx::prefetch_tmap(&tmap_h);
  }
  pdl_begin();
  KernelClock* const clk = p.clock_slot >= 0 ? &g_kernel_clocks[p.clock_slot] : nullptr;
  clock_begin(clk);
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, DK_TMEM_COLS);
    ptx::tmem_relinquish();
  }

  // ---------------------------------------------------------------- phase 0: routing
  if (p.logits == nullptr) {
    for (int s = threadIdx.x; s < kDecodeMaxSlots; s += blockDim.x) {
      s_ids[s] = s < S ? p.ids[s] : -1;
      s_w[s] = s < S ? p.wts[s] : 0.f;
    }
  } else {
    for (int s = S + threadIdx.x; s < kDecodeMaxSlots; s += blockDim.x) {
      s_ids[s] = -1;
      s_w[s] = 0.f;
    }
    // warp w routes tokens w, w + 6, w + 12 (those below T): all its logit
    // rows are loaded before the selection, so their loads overlap, and its
    // tokens are selected together (interleaved reduction chains)
    constexpr int kWarps = NUM_THREADS / 32;
    constexpr int kRounds = (kDecodeMaxTokens + kWarps - 1) / kWarps;
    const int nt = warp < p.T ? (p.T - 1 - warp) / kWarps + 1 : 0;
    float lv[kRounds][8];
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      if (r >= nt) break;
      const size_t off = (size_t)(warp + kWarps * r) * p.E;
      if (p.logits_dtype == MOE_F32)
        route_load<float, 8>(static_cast<const float*>(p.logits) + off, p.E, lane, lv[r]);
      else if (p.logits_dtype == MOE_BF16)
        route_load<__nv_bfloat16, 8>(static_cast<const __nv_bfloat16*>(p.logits) + off, p.E, lane, lv[r]);
      else
        route_load<__half, 8>(static_cast<const __half*>(p.logits) + off, p.E, lane, lv[r]);
    }
    int rid[kRounds];
    float rw[kRounds];
    auto select = [&](auto n_tag) {
      constexpr int N = decltype(n_tag)::value;
      float v[N][8];
      int id[N];
      float wt[N];
#pragma unroll
      for (int r = 0; r < N; ++r)
#pragma unroll
        for (int i = 0; i < 8; ++i) v[r][i] = lv[r][i];
      route_select<N, 8>(v, p.E, p.k, p.sigmoid, p.renormalize, lane, id, wt);
#pragma unroll
      for (int r = 0; r < N; ++r) {
        rid[r] = id[r];
        rw[r] = wt[r];
      }
    };
    static_assert(kRounds == 3, "phase-0 routing selects 1 to 3 tokens per warp");
    if (nt == 1) select(std::integral_constant<int, 1>{});
    else if (nt == 2) select(std::integral_constant<int, 2>{});
    else if (nt == 3) select(std::integral_constant<int, 3>{});
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int t = warp + kWarps * r;
      if (r < nt && lane < p.k) {
        s_ids[t * p.k + lane] = rid[r];
        s_w[t * p.k + lane] = rw[r];
        if (blockIdx.x == 0) {
          p.ids_out[t * p.k + lane] = rid[r];
          p.wts_out[t * p.k + lane] = rw[r];
        }
      }
    }
  }
  __syncthreads();
  // slot s is the first of its expert if no earlier slot has the same valid
  // id (its key: the id; other slots: a key above every id); its tile = the
  // number of keys below its id. Slot tables are read four at a time.
  if (threadIdx.x < kDecodeMaxSlots) {
    const int s = threadIdx.x, id = s_ids[s];
    bool first = id >= 0 && id < p.E;
    const int4* v = reinterpret_cast<const int4*>(s_ids);
    for (int j4 = 0; first && 4 * j4 < s; ++j4) {  // the earlier slots
      const int4 q = v[j4];
      const int j = 4 * j4;
      first = !((q.x == id) | ((q.y == id) & (j + 1 < s)) | ((q.z == id) & (j + 2 < s)) | ((q.w == id) & (j + 3 < s)));
    }
    s_key[s] = first ? id : 0x7FFFFFFF;
  }
  if (threadIdx.x == 0)  // read once per CTA, before any of its threads arrives on the counter
    *s_gen = *(volatile unsigned int*)&g_decode_bar_gen;
  __syncthreads();
  int is_first = 0;
  if (threadIdx.x < S && s_key[threadIdx.x] != 0x7FFFFFFF) {
    const int key = s_key[threadIdx.x];
    const int4* f = reinterpret_cast<const int4*>(s_key);
    int rank = 0;
    for (int j4 = 0; 4 * j4 < S; ++j4) {
      const int4 q = f[j4];
      rank += (q.x < key) + (q.y < key) + (q.z < key) + (q.w < key);
    }
    s_act[rank] = key;
    is_first = 1;
  }
  ptx::tc_fence_before();
  const int A = __syncthreads_count(is_first);  // active experts (also the barrier for s_act)
  // cluster launch: every CTA's reduction barrier is initialised before any
  // peer arrives on it (the epilogue warps wait before phase 1, the others
  // at the end)
  if (p.cluster_sp > 0) ptx::cluster_arrive();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // this launch's tag for the tagged counts: the launch generation, the same
  // for every CTA of the launch, different for every launch
  const unsigned int gen = *s_gen;
  const unsigned long long tag = ((unsigned long long)gen << 32) | 0x9e370000ull;
  const unsigned int h_total = (unsigned int)p.nf1 * 4;  // (feature tile, warp) groups of one tile's h
  const P1Plan plan1(A * p.nf1, p.kb1, (int)gridDim.x, p.cluster_sp);
  const int items2 = A * p.nf2;
  const int stages2 = (p.kb2 + 1) / 2;                        // two w2 K blocks per stage

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_par[DK_STAGES];
      for (int i = 0; i < DK_STAGES; ++i) last_par[i] = -1;
      bool ok = true;
      auto advance = [&]() {
        last_par[stage] = (int)phase;
        if (++stage == DK_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      };
      // phase 1: gate + up weight tiles and the x box of each K block
      P1Plan::Iter seg1(plan1, blockIdx.x);
      int u1, kb0, kb1;
      while (ok && seg1.next(u1, kb0, kb1)) {
        const int m = u1 / p.nf1, f = u1 % p.nf1;
        const int e = s_act[m];
        const int wrow = e * 2 * p.I + f * SW_FEAT;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + stage * DK_STAGE;
          const int kx = kb * kElems;
          ptx::mbar_arrive_expect_tx(&full[stage], DK_STAGE_A + kDecodeMaxTokens * ROW_BYTES);
          ptx::tma_load_2d(st, &tmap_w13, &full[stage], kx, wrow);
          ptx::tma_load_2d(st + SW_A_TILE, &tmap_w13, &full[stage], kx, wrow + p.I);
          ptx::tma_load_2d(st + DK_STAGE_A, &tmap_x, &full[stage], kx, 0);
          advance();
        }
      }
      // the first phase-2 stages' weights ahead of h (they do not depend on
      // it); a slot is free once its phase-1 MMAs are done, so these waits
      // never depend on other CTAs. At most one ring's worth.
      int pend_stage[DK_STAGES], pend_kb[DK_STAGES], pend_m[DK_STAGES], npend = 0;
      int it2 = blockIdx.x, kb2 = 0;  // next phase-2 stage: item it2, K blocks kb2, kb2 + 1
      while (ok && it2 < items2 && npend < DK_STAGES) {
        if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const int m = it2 / p.nf2, f = it2 % p.nf2;
        uint8_t* st = ring + stage * DK_STAGE;
        const int nkb = min(2, p.kb2 - kb2);
        ptx::mbar_arrive_expect_tx(&full[stage], nkb * (SW_A_TILE + kDecodeMaxTokens * ROW_BYTES));
        for (int j = 0; j < nkb; ++j)
          ptx::tma_load_2d(st + j * SW_A_TILE, &tmap_w2, &full[stage], (kb2 + j) * kElems,
                           s_act[m] * p.H + f * SW_FEAT);
        pend_stage[npend] = stage;
        pend_kb[npend] = kb2;
        pend_m[npend] = m;
        ++npend;
        advance();
        kb2 += 2;
        if (kb2 >= p.kb2) {
          kb2 = 0;
          it2 += gridDim.x;
        }
      }
      // tile m's h is complete once all its (feature tile, warp) groups are
      // stored, whichever CTAs computed them: a tagged count per tile. A
      // phase-2 stage's h rows are loaded once that count is full.
      int ready_m = -1;
      bool cleared = false;  // every CTA's phase-0 clears (of the counts too) are done
      auto wait_h = [&](int m) {
        if (m == ready_m) return true;
        if (!cleared && !decode_all_arrived(gen, abort_flag)) {
          raise_device_error(7);
          return false;
        }
        cleared = true;
        if (!wait_count(&p.h_ready[m], h_total, abort_flag)) {
          raise_device_error(7);
          return false;
        }
        fence_proxy_async_global();  // h was written through the generic proxy; TMA reads it
        ready_m = m;
        return true;
      };
      // every stage given an expected byte count gets its h loads, also after
      // a failed wait (then from h as it is: the kernel has failed, but the
      // stage's barrier completes, so the drain below never waits it out)
      for (int i = 0; i < npend; ++i) {
        if (ok && !wait_h(pend_m[i])) ok = false;
        uint8_t* st = ring + pend_stage[i] * DK_STAGE;
        const int nkb = min(2, p.kb2 - pend_kb[i]);
        for (int j = 0; j < nkb; ++j)
          ptx::tma_load_2d(st + DK_STAGE_A + j * kDecodeMaxTokens * ROW_BYTES, &tmap_h, &full[pend_stage[i]],
                           (pend_kb[i] + j) * kElems, pend_m[i] * kDecodeMaxTokens);
      }
      // the rest of phase 2
      while (ok && it2 < items2) {
        if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const int m = it2 / p.nf2, f = it2 % p.nf2;
        uint8_t* st = ring + stage * DK_STAGE;
        const int nkb = min(2, p.kb2 - kb2);
        ptx::mbar_arrive_expect_tx(&full[stage], nkb * (SW_A_TILE + kDecodeMaxTokens * ROW_BYTES));
        for (int j = 0; j < nkb; ++j)
          ptx::tma_load_2d(st + j * SW_A_TILE, &tmap_w2, &full[stage], (kb2 + j) * kElems,
                           s_act[m] * p.H + f * SW_FEAT);
        if (!wait_h(m)) ok = false;  // the h loads are issued regardless (see above)
        for (int j = 0; j < nkb; ++j)
          ptx::tma_load_2d(st + DK_STAGE_A + j * kDecodeMaxTokens * ROW_BYTES, &tmap_h, &full[stage],
                           (kb2 + j) * kElems, m * kDecodeMaxTokens);
        advance();
        if (!ok) break;
        kb2 += 2;
        if (kb2 >= p.kb2) {
          kb2 = 0;
          it2 += gridDim.x;
        }
      }
      if (!ok) {
        raise_device_error(1);
        *abort_flag = 1;
        // let this CTA's copies in flight land
        volatile int never = 0;
        for (int i = 0; i < DK_STAGES; ++i)
          if (last_par[i] >= 0) ptx::mbar_wait(&full[i], (uint32_t)last_par[i], &never);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      P1Plan::Iter seg1(plan1, blockIdx.x);
      int u1, kb0, kb1;
      for (; ok && seg1.next(u1, kb0, kb1); ++it) {
        const int buf = it & 1;
        if (!ptx::mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(buf * 32);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(ring + stage * DK_STAGE);
          const uint32_t b_addr = a_addr + DK_STAGE_A;
#pragma unroll
          for (int kk = 0; kk < ROW_BYTES / 32; ++kk) {
            const uint64_t bd = ptx::smem_desc_k128(b_addr + kk * 32);
            const uint32_t acc = (kb > kb0 || kk > 0) ? 1u : 0u;
            ptx::umma<KIND>(d, ptx::smem_desc_k128(a_addr + kk * 32), bd, p.idesc, acc);
            ptx::umma<KIND>(d + 16, ptx::smem_desc_k128(a_addr + SW_A_TILE + kk * 32), bd, p.idesc, acc);
          }
          ptx::umma_commit(&empty[stage]);
          if (++stage == DK_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ptx::umma_commit(&tfull[buf]);
      }
      for (int i2 = blockIdx.x; ok && i2 < items2; i2 += gridDim.x, ++it) {
        const int buf = it & 1;
        if (!ptx::mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(buf * 32);
        for (int st2 = 0; st2 < stages2; ++st2) {
          if (!ptx::mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(ring + stage * DK_STAGE);
          const uint32_t b_addr = a_addr + DK_STAGE_A;
          const int nkb = min(2, p.kb2 - 2 * st2);
          for (int j = 0; j < nkb; ++j) {
#pragma unroll
            for (int kk = 0; kk < ROW_BYTES / 32; ++kk) {
              const uint32_t acc = (st2 > 0 || j > 0 || kk > 0) ? 1u : 0u;
              ptx::umma<KIND>(d, ptx::smem_desc_k128(a_addr + j * SW_A_TILE + kk * 32),
                              ptx::smem_desc_k128(b_addr + j * kDecodeMaxTokens * ROW_BYTES + kk * 32), p.idesc, acc);
            }
          }
          ptx::umma_commit(&empty[stage]);
          if (++stage == DK_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ptx::umma_commit(&tfull[buf]);
      }
      if (!ok) {
        raise_device_error(2);
        *abort_flag = 1;
      }
      ptx::umma_commit(drain);
      volatile int never = 0;
      if (!ptx::mbar_wait(drain, 0, &never)) raise_device_error(4);
    }
  } else {
    // ------------------------------------------------------------ epilogue (128 threads)
    const int q = warp & 3;
    const int fit = q * 32 + lane;
    const int et = threadIdx.x - 64;  // 0..127
    // phase-0 work of the epilogue warps, done before the CTA arrives on the
    // launch counter (so before any CTA's phase-2 add): distinct valid experts
    // per token (the adds its output groups wait for), the fp32 accumulator
    // and group counts cleared, zero output rows for tokens with no valid slot
    if (warp == 2 && lane < p.T) {
      int c = 0;
      for (int j = 0; j < p.k; ++j) {
        const int id = s_ids[lane * p.k + j];
        bool first = id >= 0 && id < p.E;
        for (int q2 = 0; first && q2 < j; ++q2) first = s_ids[lane * p.k + q2] != id;
        c += first;
      }
      s_kd[lane] = c;
    }
    const int64_t estride = (int64_t)gridDim.x * 128;
    for (int64_t i = (int64_t)blockIdx.x * 128 + et; i < (int64_t)p.T * p.H; i += estride) p.y32[i] = 0.f;
    for (int64_t i = (int64_t)blockIdx.x * 128 + et; i < (int64_t)p.T * p.nf2 * 4; i += estride) p.conv_cnt[i] = 0;
    for (int64_t i = (int64_t)blockIdx.x * 128 + et; i < A; i += estride) p.h_ready[i] = 0;
    __threadfence();
    asm volatile("bar.sync 1, 128;" ::: "memory");  // s_kd complete, clears fenced (epilogue warps only)
    if (et == 0) decode_launch_arrive(gridDim.x);
    for (int t = 0; t < p.T; ++t)
      if (s_kd[t] == 0)
        for (int64_t i = (int64_t)blockIdx.x * 128 + et; i < p.H; i += estride)
          store1_out(p.y, p.dtype, (int64_t)t * p.H + i, 0.f);
    bool ok = true;
    bool cleared = false;  // (lane 0) every CTA's phase-0 clears are done
    if (p.cluster_sp > 0) ptx::cluster_wait();  // the cluster's reduction barriers exist
    int it = 0;
    P1Plan::Iter seg1(plan1, blockIdx.x);
    int u1, kb0, kb1;
    for (; seg1.next(u1, kb0, kb1); ++it) {
      const int m = u1 / p.nf1, f = u1 % p.nf1;
      int b_first, b_last;
      plan1.ctas(u1, b_first, b_last);
      const int buf = it & 1;
      const bool w_ok = ptx::mbar_wait(&tfull[buf], (it >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      uint32_t g[16], u[16];
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 32);
      ptx::tmem_ld16(tb, g);
      ptx::tmem_ld16(tb + 16, u);
      ptx::tmem_ld_wait();
      ptx::tc_fence_before();
      ptx::mbar_arrive(&tempty[buf]);
      const int feat = f * SW_FEAT + fit;
      const bool feat_ok = feat < p.I;
      if (b_last > b_first && p.cluster_sp > 0) {
        // the unit's K splits are the CTAs of this cluster: the others send
        // their sums to the leader's shared memory, the leader adds them in
        // split order, applies SwiGLU and stores and counts the features
        const uint32_t crank = ptx::cluster_ctarank();
        if (crank > 0) {
          const uint32_t base = ptx::mapa(ptx::smem_u32(s_red), 0);
          const int slot = ((int)(crank - 1) * 128 + fit) * 2 * p.T;
#pragma unroll
          for (int t = 0; t < kDecodeMaxTokens; ++t) {
            if (t < p.T) {
              ptx::st_cluster_f32(base + 4u * (uint32_t)(slot + t), acc_value<KIND>(g[t]));
              ptx::st_cluster_f32(base + 4u * (uint32_t)(slot + p.T + t), acc_value<KIND>(u[t]));
            }
          }
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa(ptx::smem_u32(red_bar), 0));
          continue;
        }
        const bool r_ok = ptx::mbar_wait_cluster(red_bar, 0, abort_flag);
        if (!__all_sync(0xffffffffu, r_ok)) {
          if (lane == 0) raise_device_error(7);
          ok = false;
          break;
        }
        if (feat_ok) {
#pragma unroll
          for (int t = 0; t < kDecodeMaxTokens; ++t) {
            if (t < p.T) {
              float gs = acc_value<KIND>(g[t]), us = acc_value<KIND>(u[t]);
              for (int s2 = 1; s2 < p.cluster_sp; ++s2) {
                const int slot = ((s2 - 1) * 128 + fit) * 2 * p.T;
                gs += s_red[slot + t];
                us += s_red[slot + p.T + t];
              }
              store1_out(p.h, p.dtype, ((int64_t)m * kDecodeMaxTokens + t) * p.I + feat, silu_mul(gs, us));
            }
          }
        }
      } else if (b_last > b_first) {
        const int unit = u1;
        constexpr size_t kSplit = 2 * SW_FEAT * kDecodeMaxTokens;  // floats per partial slot
        float* mine = p.partial + (size_t)plan1.slot(unit, blockIdx.x) * kSplit + fit * kDecodeMaxTokens;
        if (feat_ok) {
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            *reinterpret_cast<float4*>(mine + j) = make_float4(acc_value<KIND>(g[j]), acc_value<KIND>(g[j + 1]),
                                                               acc_value<KIND>(g[j + 2]), acc_value<KIND>(g[j + 3]));
            *reinterpret_cast<float4*>(mine + SW_FEAT * kDecodeMaxTokens + j) =
                make_float4(acc_value<KIND>(u[j]), acc_value<KIND>(u[j + 1]), acc_value<KIND>(u[j + 2]),
                            acc_value<KIND>(u[j + 3]));
          }
        }
        // the last segment of the unit to finish (per warp: its 32 features)
        // adds the partials in K order and applies SwiGLU
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = tagged_count_last(&p.split_cnt[unit * 4 + q], tag, (unsigned)(b_last - b_first + 1));
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last < 0) {
          ok = false;
          break;
        }
        if (last && feat_ok) {
          __threadfence();
          const int nseg = b_last - b_first + 1;
          for (int t = 0; t < p.T; ++t) {
            float gs = 0.f, us = 0.f;
            for (int j0 = 0; j0 < nseg; j0 += 4) {  // four segments' loads in flight, added in K order
              float gp[4], up[4];
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                gp[jj] = 0.f;
                up[jj] = 0.f;
                if (j0 + jj < nseg) {
                  const float* src = p.partial + (size_t)plan1.slot(unit, b_first + j0 + jj) * kSplit +
                                     fit * kDecodeMaxTokens + t;
                  gp[jj] = __ldcg(src);
                  up[jj] = __ldcg(src + SW_FEAT * kDecodeMaxTokens);
                }
              }
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                gs += gp[jj];
                us += up[jj];
              }
            }
            store1_out(p.h, p.dtype, ((int64_t)m * kDecodeMaxTokens + t) * p.I + feat, silu_mul(gs, us));
          }
        }
        if (!last) continue;  // the unit's last segment stores and counts this warp's features
      } else if (feat_ok) {
#pragma unroll
        for (int t = 0; t < kDecodeMaxTokens; ++t)
          if (t < p.T)
            store1_out(p.h, p.dtype, ((int64_t)m * kDecodeMaxTokens + t) * p.I + feat,
                       silu_mul(acc_value<KIND>(g[t]), acc_value<KIND>(u[t])));
      }
      // this warp's 32 features of tile m are stored: count them (once every
      // CTA has cleared its part of the counts)
      __threadfence();
      __syncwarp();
      int cnt_ok = 1;
      if (lane == 0) {
        if (!cleared && !decode_all_arrived(gen, abort_flag)) {
          raise_device_error(7);
          cnt_ok = 0;
        } else {
          cleared = true;
          atomicAdd(&p.h_ready[m], 1u);
        }
      }
      if (!__shfl_sync(0xffffffffu, cnt_ok, 0)) {
        ok = false;
        break;
      }
    }
    // phase 2: weighted adds into the fp32 accumulator, once every CTA has
    // cleared its part of it (all arrived on the launch counter)
    if (ok && blockIdx.x < items2) {
      int arrived = 1;
      if (lane == 0 && !cleared) arrived = decode_all_arrived(gen, abort_flag);
      if (!__shfl_sync(0xffffffffu, arrived, 0)) {
        if (lane == 0) raise_device_error(7);
        ok = false;
      }
    }
    for (int i2 = blockIdx.x; ok && i2 < items2; i2 += gridDim.x, ++it) {
      const int m = i2 / p.nf2, f = i2 % p.nf2;
      const int buf = it & 1;
      const bool w_ok = ptx::mbar_wait(&tfull[buf], (it >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      uint32_t v[16];
      ptx::tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 32), v);
      ptx::tmem_ld_wait();
      ptx::tc_fence_before();
      ptx::mbar_arrive(&tempty[buf]);
      const int feat = f * SW_FEAT + fit;
      const bool feat_ok = feat < p.H;
      const int e = s_act[m];
      // lane t < T: token t's routing weight for expert e (summed if it
      // lists e twice), broadcast to the warp below
      float my_w = 0.f;
      if (lane < p.T)
        for (int j = 0; j < p.k; ++j)
          if (s_ids[lane * p.k + j] == e) my_w += s_w[lane * p.k + j];
#pragma unroll
      for (int t = 0; t < kDecodeMaxTokens; ++t) {
        if (t >= p.T) break;
        const float w = __shfl_sync(0xffffffffu, my_w, t);
        if (w != 0.f && feat_ok) red_add1(p.y32 + (int64_t)t * p.H + feat, w * acc_value<KIND>(v[t]));
      }
      // count this warp's adds per token; the warp completing a (token,
      // group) converts its 32 features
      __threadfence();
      __syncwarp();
      bool done = false;
      if (lane < p.T && my_w != 0.f)
        done = atomicAdd(&p.conv_cnt[lane * p.nf2 * 4 + f * 4 + q], 1) == s_kd[lane] - 1;
      unsigned todo = __ballot_sync(0xffffffffu, done);
      if (todo) __threadfence();
      while (todo) {
        const int t = __ffs(todo) - 1;
        todo &= todo - 1;
        if (feat_ok) store1_out(p.y, p.dtype, (int64_t)t * p.H + feat, __ldcg(p.y32 + (int64_t)t * p.H + feat));
      }
    }
    if (!ok) {
      if (lane == 0) raise_device_error(3);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  clock_end(clk);
  if (p.cluster_sp > 0) {
    if (warp < 2) ptx::cluster_wait();  // the producer and MMA warps' wait on the barrier after phase 0
    ptx::cluster_sync();                // no CTA leaves while a peer may still write its shared memory
  }
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, DK_TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side

std::atomic<int> g_decode_fused{1};  // MOE_OPT_DECODE_FUSED

constexpr size_t kDecodeSmem =
    1024 + (size_t)DK_STAGES * DK_STAGE + 256 + 4 * kDecodeMaxSlots * 4 + 16 * 4 + kDecodeRedBytes + 16;

struct DecodeWs {
  int max_tiles, nf1, nf2, kb1, kb2, grid;  // grid: CTAs of the launch
  int sp1;  // gate_up K splits when every routed expert is distinct
  size_t h, partial, split_cnt, h_ready, y32, conv_cnt, bytes;
};

DecodeWs decode_ws(int64_t T, int k, int E, int64_t H, int64_t I, int dtype) {
  DecodeWs w;
  const int es = dtype_size(dtype);
  w.max_tiles = (int)std::min<int64_t>(E, T * k);
  w.nf1 = (int)ceil_div(I, SW_FEAT);
  w.nf2 = (int)ceil_div(H, SW_FEAT);
  w.kb1 = (int)ceil_div(H * es, ROW_BYTES);
  w.kb2 = (int)ceil_div(I * es, ROW_BYTES);
  const int64_t units1 = (int64_t)w.max_tiles * w.nf1, sms = num_sms();
  // enough CTAs for the gate_up units (K-split while they fill at most half
  // the SMs, with at most as many splits as the kernel will choose) and the
  // down items, at most one per SM (all resident)
  const int64_t sp = (2 * units1 <= sms)
                         ? std::max<int64_t>(1, std::min<int64_t>({sms / units1, (int64_t)w.kb1 / 4, kDecodeMaxSplits}))
                         : 1;
  w.grid = (int)std::min<int64_t>(sms, std::max<int64_t>(units1 * sp, (int64_t)w.max_tiles * w.nf2));
  w.sp1 = (int)sp;
  size_t off = 0;
  auto take = [&](size_t b) {
    const size_t o = off;
    off = align_up(off + b, 256);
    return o;
  };
  w.h = take((size_t)w.max_tiles * kDecodeMaxTokens * I * es);
  w.partial = take((size_t)w.grid * 2 * SW_FEAT * kDecodeMaxTokens * 4);  // one slot per CTA
  w.split_cnt = take((size_t)units1 * 4 * sizeof(unsigned long long));
  w.h_ready = take((size_t)w.max_tiles * sizeof(unsigned int));
  w.y32 = take((size_t)T * H * 4);
  w.conv_cnt = take((size_t)T * w.nf2 * 4 * sizeof(int32_t));
  w.bytes = off;
  return w;
}

}  // namespace

bool decode_fused_fits(int64_t T, int k, int E, int64_t H, int64_t I, int x_dtype, int w_dtype) {
  return g_decode_fused.load() != 0 && T >= 1 && T <= kDecodeMaxTokens && T * k <= kDecodeMaxSlots && E >= 1 &&
         E <= (1 << 20) && x_dtype == w_dtype && (x_dtype == MOE_BF16 || x_dtype == MOE_F16) && H % 8 == 0 &&
         I % 8 == 0 && (int64_t)E * 2 * I < (int64_t(1) << 31) && (int64_t)E * H < (int64_t(1) << 31);
}

size_t decode_fused_workspace(int64_t T, int k, int E, int64_t H, int64_t I, int dtype) {
  return decode_ws(T, k, E, H, I, dtype).bytes;
}

bool decode_route_fits(int E, int k, int logits_dtype) {
  return E <= kDecodeRouteMaxExperts && k <= 32 &&
         (logits_dtype == MOE_F32 || logits_dtype == MOE_BF16 || logits_dtype == MOE_F16);
}

int decode_fused(const void* x, int dtype, int64_t T, int64_t H, const void* w13, const void* w2, int E, int64_t I,
                 const float* topk_weights, const int32_t* topk_ids, int k, void* y, void* workspace,
                 size_t workspace_bytes, cudaStream_t st, const DecodeRouting* route) {
  MOE_CHECK_ARG(decode_fused_fits(T, k, E, H, I, dtype, dtype), "decode_fused: batch outside the one-launch path");
  MOE_CHECK_ARG(x && w13 && w2 && y && (route ? route->logits && route->ids_out && route->wts_out
                                                : topk_weights && topk_ids),
                "decode_fused: NULL pointer");
  MOE_CHECK_ARG(!route || decode_route_fits(E, k, route->dtype), "decode_fused: routing outside the one-launch path");
  MOE_CHECK_ARG((uintptr_t)x % 16 == 0 && (uintptr_t)w13 % 16 == 0 && (uintptr_t)w2 % 16 == 0,
                "decode_fused: pointers must be 16-byte aligned");
  const DecodeWs w = decode_ws(T, k, E, H, I, dtype);
  if (workspace_bytes < w.bytes || !workspace)
    return set_error(MOE_ERR_WORKSPACE, "decode_fused: workspace %zu < %zu bytes", workspace_bytes, w.bytes);
  char* ws = static_cast<char*>(workspace);
  CUtensorMap t13, t2, tx, th;
  MOE_TRY(make_tmap(&t13, w13, dtype, H, (uint64_t)E * 2 * I, SW_FEAT));
  MOE_TRY(make_tmap(&t2, w2, dtype, I, (uint64_t)E * H, SW_FEAT));
  MOE_TRY(make_tmap(&tx, x, dtype, H, T, kDecodeMaxTokens));
  MOE_TRY(make_tmap(&th, ws + w.h, dtype, I, (uint64_t)w.max_tiles * kDecodeMaxTokens, kDecodeMaxTokens));
  DecodeParams p{};
  p.T = (int)T;
  p.k = k;
  p.E = E;
  p.I = (int)I;
  p.H = (int)H;
  p.nf1 = w.nf1;
  p.nf2 = w.nf2;
  p.kb1 = w.kb1;
  p.kb2 = w.kb2;
  p.max_tiles = w.max_tiles;
  p.idesc = (make_idesc(dtype, SW_FEAT) & ~(0x3Fu << 17)) | ((uint32_t)(kDecodeMaxTokens >> 3) << 17);
  p.ids = topk_ids;
  p.wts = topk_weights;
  p.h = ws + w.h;
  p.partial = reinterpret_cast<float*>(ws + w.partial);
  p.split_cnt = reinterpret_cast<unsigned long long*>(ws + w.split_cnt);
  p.h_ready = reinterpret_cast<unsigned int*>(ws + w.h_ready);
  p.y32 = reinterpret_cast<float*>(ws + w.y32);
  p.conv_cnt = reinterpret_cast<int32_t*>(ws + w.conv_cnt);
  p.y = y;
  p.dtype = dtype;
  p.clock_slot = g_kernel_clocks_on.load() ? MOE_CLOCK_GATE_UP : -1;
  if (route) {
    p.logits = route->logits;
    p.logits_dtype = route->dtype;
    p.sigmoid = route->sigmoid;
    p.renormalize = route->renormalize;
    p.ids_out = route->ids_out;
    p.wts_out = route->wts_out;
  }
  int64_t grid = w.grid;
  auto kfn = moe_decode_kernel<0>;
  MOE_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmem));
  // K-split gate_up units reduce through distributed shared memory when each
  // unit's splits can form one cluster, the other splits' sums fit the
  // leader's buffer and every cluster of the grid can be resident at once
  // (the kernel's CTAs wait on one another). The split count is the largest,
  // up to the one without clusters, whose clusters all fit: at one token of
  // the Qwen3 layer 48 units need 48 clusters, three-CTA clusters fit 45 at
  // once and two-CTA clusters 74, so it runs two splits per unit (measured
  // 27.6 vs 28.5 µs for three splits reduced through global memory).
  int cluster = 0;
  const int64_t sms = num_sms(), units_ub = (int64_t)w.max_tiles * w.nf1, items2_ub = (int64_t)w.max_tiles * w.nf2;
  for (int spc = (g_decode_fused.load() == 1) ? w.sp1 : 0; spc >= 2 && !cluster; --spc) {
    if ((int64_t)(spc - 1) * T * 128 * 2 * 4 > kDecodeRedBytes) continue;
    const int64_t gc = ceil_div(std::min<int64_t>(sms, std::max<int64_t>(units_ub * spc, items2_ub)), (int64_t)spc) * spc;
    if (gc > sms) continue;
    cudaLaunchConfig_t occ = {};
    cudaLaunchAttribute ca[1];
    occ.gridDim = dim3((unsigned)gc);
    occ.blockDim = dim3(NUM_THREADS);
    occ.dynamicSmemBytes = kDecodeSmem;
    ca[0].id = cudaLaunchAttributeClusterDimension;
    ca[0].val.clusterDim.x = (unsigned)spc;
    ca[0].val.clusterDim.y = 1;
    ca[0].val.clusterDim.z = 1;
    occ.attrs = ca;
    occ.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &occ) != cudaSuccess) {
      (void)cudaGetLastError();  // not fatal: the launch runs without clusters
      break;
    }
    if ((int64_t)n * spc >= gc) {
      cluster = spc;
      grid = gc;
    }
  }
  p.cluster_sp = cluster;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = kDecodeSmem;
  cfg.stream = st;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  MOE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, t13, t2, tx, th, p));
  MOE_LAUNCH_CHECK("moe_decode_kernel");
  return MOE_OK;
}

}  // namespace moe
