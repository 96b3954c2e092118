// Grouped MoE GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One persistent, warp-specialised kernel template serves both GEMMs of the
// expert MLP:
//   GEMM1 (SWIGLU=true):  h = silu(a . w_gate) * (a . w_up)   (+ w8a8 dequant)
//   GEMM2 (SWIGLU=false): out = h . w2 with three epilogues (row store,
//                         weighted scatter-add combine, row scatter)
// Reference kernels replaced: _grouped_gemm1_swiglu_kernel /
// _grouped_gemm2_kernel (partially_fused_moe_mlp_triton.py:59-162) and the two
// halves of _fused_moe_mlp_kernel (fused_moe_mlp_triton.py:35-88).
//
// CTA layout (192 threads, one CTA per SM; two variants, see Cfg):
//   warp 0      TMA producer, 128B-swizzled ring in shared memory. One CTA per
//               tile: A (128 rows x 128 B) + B (256 rows x 128 B) per stage,
//               4 stages. CTA pair: each CTA its own 128 A rows + half of B
//               (128 rows), 6 stages, both counted on the leader's barrier.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128 or,
//               for a pair, M=256 / M=128; N=256; K=32 bytes per instruction)
//               into one of two 256-column fp32/int32 accumulators
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32*(w%4)..+31), fused SwiGLU / dequant / combine, stores
// The two accumulators let the epilogue of tile i overlap the MMAs of tile
// i+1. Tiles are visited expert-major (all tiles of expert e, in bands of 16
// M-tiles x all N-tiles), so CTAs running at the same time share weight
// tiles through L2 and each expert's weights stream from HBM about once.
#include <cuda.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "ptx.cuh"

namespace moe {

__device__ int g_moe_device_error = 0;
__device__ KernelClock g_kernel_clocks[MOE_NUM_CLOCKS];

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int ROW_BYTES = 128;             // K bytes per stage (one 128B swizzle atom)
constexpr int A_BYTES = BM * ROW_BYTES;    // 16 KiB
constexpr int NUM_THREADS = 192;
constexpr int GROUP_M = 16;
constexpr int TMEM_COLS = 512;             // 2 accumulators x 256 columns
constexpr int BAR_BYTES = 256;             // barriers + tmem slot + abort flag
constexpr int MAX_GEMM_EXPERTS = 1024;
constexpr int STAGE_ROW_BYTES = 144;       // 128 B of a row + 16 B pad (conflict-free)
constexpr int STAGE_WARP_BYTES = 32 * STAGE_ROW_BYTES;
constexpr int EPI_STAGE_BYTES = 4 * STAGE_WARP_BYTES;  // one area per epilogue warp (down GEMM)
constexpr int kEpiScaleCols = 256;                     // int8 column scales of one N tile
constexpr int EPI_SCALE_BYTES = 4 * 2 * kEpiScaleCols * 4;  // int8: two tiles' scales per epilogue warp

__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_moe_device_error, 0, code); }

struct Params {
  int E;
  int num_kb;             // K blocks of 128 bytes
  int n_tiles;            // tiles along N
  int n_valid;            // valid output columns (I for GEMM1, H for GEMM2)
  int b_rows_per_expert;  // rows of B per expert (2I or H)
  int inter;              // GEMM1: row offset of the up half within an expert
  uint32_t idesc;         // tcgen05 instruction descriptor
  uint32_t idesc_half;    // CTA pair: descriptor of the M=128 MMA (64 rows per CTA) for an odd last tile
  int half_units;         // CTA pair: run each expert's odd last tile as an M=128 pair MMA
  const int32_t* table;
  int max_tiles;
  int64_t a_rows;
  int epi;
  void* out;
  int out_dtype;
  int64_t ldo;
  int64_t out_rows;
  const float* a_scale;
  const float* b_scale;
  const int32_t* row_map;
  const float* row_weight;
  int top_k;
  void* const* peer_out;  // kEpiScatterPeer: device array of per-rank output bases
  int num_peers;
  int band_tiles;         // M tiles per band of the expert-major raster
  int stream_k;           // split the (unit, K block) space evenly (additive epilogues only)
  int clock_slot;         // kernel clock class (MOE_OPT_KERNEL_CLOCKS), -1 = off
};

// The work of one CTA (or CTA pair): whole units t = gid, gid + n, ... in
// raster order for every full wave of n units; with stream-K the units of the
// partial last wave are then split along K, each of the n groups taking an
// equal contiguous share of their (unit, K block) space, so no group idles
// while others finish the tail. Segments are (unit t, K blocks [kb0, kb1)).
struct SegIter {
  bool sk;
  int t, stride, num_kb, full_end;
  int64_t w, w1;
  __device__ __forceinline__ SegIter(bool stream_k, int gid, int ngroups, int total_units, int kb)
      : sk(stream_k), t(gid), stride(ngroups), num_kb(kb), full_end(total_units), w(0), w1(0) {
    if (sk) {
      full_end = total_units / ngroups * ngroups;  // units run whole
      const int64_t tail = (int64_t)(total_units - full_end) * kb;
      w = (int64_t)full_end * kb + tail * gid / ngroups;
      w1 = (int64_t)full_end * kb + tail * (gid + 1) / ngroups;
    }
  }
  __device__ __forceinline__ bool next(int& tt, int& kb0, int& kb1) {
    if (t < full_end) {
      tt = t;
      kb0 = 0;
      kb1 = num_kb;
      t += stride;
      return true;
    }
    if (!sk || w >= w1) return false;
    tt = (int)(w / num_kb);
    kb0 = (int)(w % num_kb);
    kb1 = (int)min((int64_t)num_kb, kb0 + (w1 - w));
    w += kb1 - kb0;
    return true;
  }
};

// Scheduling unit t -> (unit u, n tile, expert e) in expert-major order:
// the units of expert e in bands of `group` units, each band swept over all
// n tiles, so concurrently running CTAs share weight tiles through L2.
__device__ __forceinline__ void decode_unit(int t, const int32_t* s_u, int E, int NT, int group, int& u, int& n,
                                            int& e) {
  int lo = 0, hi = E;  // invariant: s_u[lo]*NT <= t < s_u[hi]*NT
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s_u[mid] * NT <= t) lo = mid;
    else hi = mid;
  }
  e = lo;
  const int mt = s_u[e + 1] - s_u[e];
  const int local = t - s_u[e] * NT;
  const int band = local / (group * NT);
  const int m0 = band * group;
  const int bsz = min(group, mt - m0);
  const int rem = local - band * group * NT;
  n = rem / bsz;
  u = s_u[e] + m0 + rem % bsz;
}

__host__ __device__ constexpr int align_up16(int v) { return (v + 15) & ~15; }

// silu(g) * u with the fast divide: for g below about -87, 1 + exp(-g)
// overflows and the quotient is 0, the limit of silu there.
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// What the epilogue needs to drain one tile, fetched one tile ahead.
struct EpiMeta {
  bool live, valid, half, row_ok;
  int e, n, m, r;  // unit's expert, N tile, this CTA's M tile; this thread's row in the tile
  int32_t rstart, rcount, slot;
  int64_t grow;
  float sa, wgt;   // int8 row scale, routing weight
  float sc[8];     // int8: this lane's 8 of the N tile's column scales
};

// Stores 8 consecutive fp32 values as the output dtype (16- or 32-byte store).
__device__ __forceinline__ void store8_out(void* base, int dtype, int64_t idx, const float* v) {
  if (dtype == MOE_BF16) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(base) + idx) = u;
  } else if (dtype == MOE_F16) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(static_cast<__half*>(base) + idx) = u;
  } else {
    float* f = static_cast<float*>(base) + idx;
    *reinterpret_cast<float4*>(f) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(f + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
}

__device__ __forceinline__ void red_add4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Row-contiguous store of this warp's 32 rows x (16 * PARTS) bytes: each lane
// packs its own row into the warp's shared-memory area, then consecutive
// lanes write consecutive 16-byte parts of one row (32 / PARTS rows per
// instruction), which keeps remote (NVLink) and local stores in long
// segments. row_ptr: destination of this lane's row, or 0 to skip it;
// nbytes_valid: leading bytes of every row to write (a multiple of 16).
// (The SwiGLU epilogue keeps row-per-thread stores: h goes to local HBM only,
// and staging it measured slower: gate_up 1.63 vs 1.42 ms on the Mixtral layer.)
template <int PARTS>
__device__ __forceinline__ void staged_store(uint8_t* stage, const uint32_t (&packed)[PARTS * 4],
                                             unsigned long long row_ptr, int nbytes_valid, int lane) {
  uint4* mine = reinterpret_cast<uint4*>(stage + lane * STAGE_ROW_BYTES);
#pragma unroll
  for (int j = 0; j < PARTS; ++j)
    mine[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < PARTS; ++i) {
    const int c = lane + 32 * i;
    const int row = c / PARTS, part = c % PARTS;
    const unsigned long long rp = __shfl_sync(0xffffffffu, row_ptr, row);
    if (rp != 0ull && part * 16 < nbytes_valid) {
      const uint4 v = *reinterpret_cast<const uint4*>(stage + row * STAGE_ROW_BYTES + part * 16);
      *reinterpret_cast<uint4*>(reinterpret_cast<char*>(rp) + part * 16) = v;
    }
  }
  __syncwarp();
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int dtype) {
  if (dtype == MOE_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int KIND>
__device__ __forceinline__ float acc_value(uint32_t bits) {
  if constexpr (KIND == 2) return static_cast<float>(static_cast<int32_t>(bits));
  else return __uint_as_float(bits);
}

// Pipeline geometry of the two variants. A scheduling unit is one 128-row M
// tile (single CTA) or two consecutive M tiles of one expert (CTA pair). In a
// pair, the odd last tile of an expert is a half unit: one M=128 pair MMA
// (cta_group::2) whose 128 rows split 64 / 64 over the two CTAs, which runs at
// the same rate per row as the M=256 MMA (64 vs 128 cycles for N=256, K=16),
// so no CTA idles. Its accumulator layout in each CTA's tensor memory: lanes
// 0-63 hold the CTA's 64 rows x N columns [0, N/2), lanes 64-127 the same rows
// x columns [N/2, N), both at TMEM columns [0, N/2).
template <bool PAIR>
struct Cfg {
  static constexpr int kStages = PAIR ? 6 : 4;
  static constexpr int kBRows = PAIR ? BN / 2 : BN;  // B rows this CTA loads per stage
  static constexpr int kBBytes = kBRows * ROW_BYTES;
  static constexpr int kStageBytes = A_BYTES + kBBytes;
  static constexpr uint32_t kTxBytes = PAIR ? 2 * kStageBytes : kStageBytes;  // per stage, whole MMA
};

// tmap_a64: A with 64-row boxes, the MMA rows of a half unit's CTA.
// tmap_b64: B with 64-row boxes; the gate_up GEMM's half units load 64 gate
// and 64 up rows per CTA so that one thread's TMEM lane holds both.
template <int KIND, bool SWIGLU, bool PAIR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_a64, const __grid_constant__ CUtensorMap tmap_b64,
                    const Params p) {
  using C = Cfg<PAIR>;
  constexpr int S = C::kStages;
  constexpr uint32_t kHalfTxBytes = 2 * (A_BYTES / 2 + C::kBBytes);  // per stage of a half unit, both CTAs
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * C::kBBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_cum = reinterpret_cast<int32_t*>(smem + S * C::kStageBytes + BAR_BYTES);
  int32_t* s_ucum = PAIR ? s_cum + (p.E + 1) : s_cum;  // scheduling-unit prefix per expert
  uint8_t* epi_stage = smem + S * C::kStageBytes + BAR_BYTES + align_up16(2 * (p.E + 1) * 4);
  uint8_t* epi_scales = epi_stage + EPI_STAGE_BYTES;  // int8 kinds only

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const uint32_t rank = PAIR ? ptx::cluster_ctarank() : 0;
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      ptx::mbar_init(&tempty[a], (PAIR ? 2 : 1) * 4 * 32);  // epilogue threads of the whole MMA
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
    if (PAIR && p.half_units) ptx::prefetch_tmap(&tmap_a64);
    if (SWIGLU && PAIR && p.half_units) ptx::prefetch_tmap(&tmap_b64);
  }
  pdl_begin();  // the tile table and operands come from the grids before this one
  KernelClock* const clk = p.clock_slot >= 0 ? &g_kernel_clocks[p.clock_slot] : nullptr;
  clock_begin(clk);
  for (int i = threadIdx.x; i <= E; i += blockDim.x) s_cum[i] = p.table[TileTable::cum_off() + i];
  if constexpr (PAIR) {
    __syncthreads();
    if (warp == 0) {  // pairs per expert = ceil(tiles / 2), prefix-summed by one warp
      const int per = (E + 31) / 32;
      const int lo = min(E, lane * per), hi = min(E, lo + per);
      int sum = 0;
      for (int e = lo; e < hi; ++e) sum += (s_cum[e + 1] - s_cum[e] + 1) >> 1;
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      int run = incl - sum;
      for (int e = lo; e < hi; ++e) {
        s_ucum[e] = run;
        run += (s_cum[e + 1] - s_cum[e] + 1) >> 1;
      }
      if (lane == 31) s_ucum[E] = incl;
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      ptx::tmem_alloc_pair(tmem_slot, TMEM_COLS);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(tmem_slot, TMEM_COLS);
      ptx::tmem_relinquish();
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) ptx::cluster_sync();  // the leader's barriers exist before the peer signals them
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int NT = p.n_tiles;
  const int total = s_ucum[E] * NT;
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int32_t* row_start_tab = p.table + TileTable::start_off(E);
  const int32_t* row_count_tab = p.table + TileTable::count_off(E, p.max_tiles);

  const int group_units = max(1, PAIR ? p.band_tiles / 2 : p.band_tiles);
  // unit t -> (expert e, n tile, this CTA's M tile m, whether m holds rows,
  // whether the unit is a half unit: one tile split 64 / 64 over the pair)
  auto locate = [&](int t, int& e, int& n, int& m, bool& valid, bool& half) {
    int u;
    decode_unit(t, s_ucum, E, NT, group_units, u, n, e);
    if constexpr (PAIR) {
      const int m0 = s_cum[e] + 2 * (u - s_ucum[e]);
      half = p.half_units && m0 + 1 == s_cum[e + 1];
      m = half ? m0 : m0 + (int)rank;
      valid = m < s_cum[e + 1];
    } else {
      m = u;
      valid = true;
      half = false;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_par[S];
#pragma unroll
      for (int s = 0; s < S; ++s) last_par[s] = -1;
      bool ok = true;
      SegIter seg(p.stream_k != 0, unit0, ustride, total, p.num_kb);
      int t, kb_begin, kb_end;
      while (ok && seg.next(t, kb_begin, kb_end)) {
        int e, n, m;
        bool valid, half;
        locate(t, e, n, m, valid, half);
        // an empty peer half still loads a (masked) A box: the rows after the
        // expert's last tile; in a half unit each CTA's MMA rows are the first
        // 64 of its box
        const int row0 = half ? row_start_tab[m] + (int)rank * (BM / 2)
                              : (valid ? row_start_tab[m] : row_start_tab[m - 1] + BM);
        int brow;
        if constexpr (SWIGLU) {
          if (half)  // gate rows [64 r, 64 r + 64) of the N tile, then the same up rows
            brow = e * p.b_rows_per_expert + n * (BN / 2) + (int)rank * (BN / 4);
          else
            brow = e * p.b_rows_per_expert + n * (BN / 2) + ((PAIR && rank) ? p.inter : 0);
        } else {
          brow = e * p.b_rows_per_expert + n * BN + (PAIR ? (int)rank * (BN / 2) : 0);
        }
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const int kx = kb * (ROW_BYTES / (KIND == 0 ? 2 : (KIND == 1 ? 4 : 1)));
          if constexpr (PAIR) {
            // a half unit loads only its 64 MMA rows of A per CTA
            if (leader) ptx::mbar_arrive_expect_tx(&full[stage], half ? kHalfTxBytes : C::kTxBytes);
            const uint32_t bar = ptx::mapa(ptx::smem_u32(&full[stage]), 0);  // the leader's full barrier
            ptx::tma_load_2d_pair(sA + stage * A_BYTES, half ? &tmap_a64 : &tmap_a, bar, kx, row0);
            if (SWIGLU && half) {
              ptx::tma_load_2d_pair(sB + stage * C::kBBytes, &tmap_b64, bar, kx, brow);
              ptx::tma_load_2d_pair(sB + stage * C::kBBytes + C::kBBytes / 2, &tmap_b64, bar, kx, brow + p.inter);
            } else {
              ptx::tma_load_2d_pair(sB + stage * C::kBBytes, &tmap_b, bar, kx, brow);
            }
          } else {
            ptx::mbar_arrive_expect_tx(&full[stage], C::kTxBytes);
            ptx::tma_load_2d(sA + stage * A_BYTES, &tmap_a, &full[stage], kx, row0);
            if constexpr (SWIGLU) {
              ptx::tma_load_2d(sB + stage * C::kBBytes, &tmap_b, &full[stage], kx, brow);
              ptx::tma_load_2d(sB + stage * C::kBBytes + C::kBBytes / 2, &tmap_b, &full[stage], kx, brow + p.inter);
            } else {
              ptx::tma_load_2d(sB + stage * C::kBBytes, &tmap_b, &full[stage], kx, brow);
            }
          }
          last_par[stage] = (int)phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      volatile int never = 0;
      if (!ok) {
        raise_device_error(1);
        *abort_flag = 1;
        // let this CTA's copies already in flight land before it exits (in a
        // pair they are counted on the leader's barriers)
        if (!PAIR || leader)
          for (int s = 0; s < S; ++s)
            if (last_par[s] >= 0) ptx::mbar_wait(&full[s], (uint32_t)last_par[s], &never);
      } else if constexpr (PAIR) {
        // every stage this CTA filled has been released by the leader's MMA
        // commit (which also lands on this CTA's barriers) before exiting
        for (int i = 0; i < S; ++i) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, &never)) raise_device_error(4);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (the leader of a pair)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      SegIter seg(p.stream_k != 0, unit0, ustride, total, p.num_kb);
      int t, kb_begin, kb_end;
      for (; ok && seg.next(t, kb_begin, kb_end); ++it) {
        const int acc = it & 1;
        const uint32_t acc_par = (it >> 1) & 1;
        if (!ptx::mbar_wait(&tempty[acc], acc_par ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        uint32_t idesc = p.idesc;
        if constexpr (PAIR) {
          int e, n, m;
          bool valid, half;
          locate(t, e, n, m, valid, half);
          if (half) idesc = p.idesc_half;
        }
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = ptx::smem_u32(sB + stage * C::kBBytes);
#pragma unroll
          for (int k = 0; k < ROW_BYTES / 32; ++k) {
            const uint64_t ad = ptx::smem_desc_k128(a_addr + k * 32), bd = ptx::smem_desc_k128(b_addr + k * 32);
            const uint32_t accum = (kb > kb_begin || k > 0) ? 1u : 0u;
            if constexpr (PAIR) ptx::umma_pair<KIND>(d, ad, bd, idesc, accum);
            else ptx::umma<KIND>(d, ad, bd, idesc, accum);
          }
          if constexpr (PAIR) ptx::umma_commit_pair_mc(&empty[stage], 0x3);
          else ptx::umma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) ptx::umma_commit_pair_mc(&tfull[acc], 0x3);
        else ptx::umma_commit(&tfull[acc]);
      }
      if (!ok) {
        raise_device_error(2);
        *abort_flag = 1;
      }
      // all MMAs issued by this thread complete before TMEM is released
      if constexpr (PAIR) ptx::umma_commit_pair(drain);
      else ptx::umma_commit(drain);
      volatile int never = 0;
      if (!ptx::mbar_wait(drain, 0, &never)) raise_device_error(4);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const uint32_t tempty_leader[2] = {PAIR ? ptx::mapa(ptx::smem_u32(&tempty[0]), 0) : ptx::smem_u32(&tempty[0]),
                                       PAIR ? ptx::mapa(ptx::smem_u32(&tempty[1]), 0) : ptx::smem_u32(&tempty[1])};
    // The facts of the tile after the current one are fetched while the
    // current one drains, so their global-memory latency stays off the
    // drain: its tile row range and (int8) its 256 column scales as soon as
    // the tile is known, this thread's row scale / routed slot after the
    // first chunk, the slot's routing weight after the second. The column
    // scales go to this warp's shared-memory buffer (two, alternating).
    float* const s_scales = reinterpret_cast<float*>(epi_scales) + (warp - 2) * 2 * kEpiScaleCols;
    EpiMeta cur, nxt;
    auto fetch_tile = [&](EpiMeta& mt, int tt) {
      locate(tt, mt.e, mt.n, mt.m, mt.valid, mt.half);
      mt.r = mt.half ? (int)rank * (BM / 2) + (q & 1) * 32 + lane : q * 32 + lane;
      mt.rstart = mt.valid ? row_start_tab[mt.m] : 0;
      mt.rcount = mt.valid ? row_count_tab[mt.m] : 0;
      if constexpr (KIND == 2) {
        const int64_t wrow = (int64_t)mt.e * p.b_rows_per_expert;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int idx = lane + 32 * i;
          int64_t src;
          if constexpr (SWIGLU)  // [0, 128): gate scales of the tile's features, [128, 256): up scales
            src = wrow + (idx >= 128 ? p.inter : 0) + min(mt.n * (BN / 2) + (idx & 127), p.n_valid - 1);
          else
            src = wrow + min(mt.n * BN + idx, p.n_valid - 1);
          mt.sc[i] = p.b_scale[src];
        }
      }
    };
    auto fetch_rows = [&](EpiMeta& mt) {
      mt.grow = (int64_t)mt.rstart + mt.r;
      mt.row_ok = (mt.r < mt.rcount) && (mt.grow < p.a_rows);
      mt.sa = 1.f;
      if constexpr (KIND == 2) mt.sa = mt.row_ok ? p.a_scale[mt.grow] : 0.f;
      mt.slot = (!SWIGLU && p.epi != MOE_EPI_STORE_ROWS && mt.row_ok) ? p.row_map[mt.grow] : -1;
    };
    auto fetch_weight = [&](EpiMeta& mt) {
      mt.wgt = (!SWIGLU && p.epi != MOE_EPI_STORE_ROWS && p.epi != kEpiScatterPeer && mt.slot >= 0 && p.row_weight)
                   ? p.row_weight[mt.slot]
                   : 1.f;
    };
    auto stage_scales = [&](const EpiMeta& mt, int buf) {
      if constexpr (KIND == 2) {
#pragma unroll
        for (int i = 0; i < 8; ++i) s_scales[buf * kEpiScaleCols + lane + 32 * i] = mt.sc[i];
        __syncwarp();
      }
    };

    int it = 0;
    bool ok = true;
    SegIter seg(p.stream_k != 0, unit0, ustride, total, p.num_kb);
    int t, kb_begin, kb_end;
    cur.live = seg.next(t, kb_begin, kb_end);
    if (cur.live) {
      fetch_tile(cur, t);
      fetch_rows(cur);
      fetch_weight(cur);
      stage_scales(cur, 0);
    }
    for (; cur.live; ++it) {
      nxt.live = seg.next(t, kb_begin, kb_end);
      if (nxt.live) fetch_tile(nxt, t);
      // after chunk c of this tile: the next tile's dependent loads
      auto chunk_done = [&](int c) {
        if (nxt.live) {
          if (c == 0) fetch_rows(nxt);
          else if (c == 1) fetch_weight(nxt);
        }
      };
      const int acc = it & 1;
      const uint32_t acc_par = (it >> 1) & 1;
      bool w_ok = ptx::mbar_wait(&tfull[acc], acc_par, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const int n = cur.n;
      const bool half = cur.half;
      const int64_t grow = cur.grow;
      const bool row_ok = cur.row_ok;
      const float sa = cur.sa;
      const float* sc = s_scales + (it & 1) * kEpiScaleCols;  // this tile's column scales (int8)
      // TMEM column 0 of this thread's lane; the row and first column it
      // holds relative to the unit's N tile follow from the lane quarter
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);

      if constexpr (SWIGLU) {
        // whole unit: gate at TMEM columns [0, 128), up at [128, 256), 128
        // features; half unit: this lane's 64 features, gate at [0, 64), up
        // at [64, 128)
        const int nchunk = half ? 2 : 4;
        const int up_col = half ? BN / 4 : BN / 2;
        const int lbase = half ? (q >> 1) * (BN / 4) : 0;  // first feature of this lane within the N tile
        const int cbase = n * (BN / 2) + lbase;
#pragma unroll 1
        for (int c = 0; c < nchunk; ++c) {
          uint32_t g[32], u[32];
          ptx::tmem_ld32(tbase + c * 32, g);
          ptx::tmem_ld32(tbase + up_col + c * 32, u);
          ptx::tmem_ld_wait();
          const int col0 = cbase + c * 32;
          if (row_ok && col0 < p.n_valid) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int cj = col0 + 8 * j;
              if (cj < p.n_valid) {
                float gs[8], us[8];
                if constexpr (KIND == 2) {
                  const int l = lbase + c * 32 + 8 * j;  // feature within the N tile
                  *reinterpret_cast<float4*>(gs) = *reinterpret_cast<const float4*>(sc + l);
                  *reinterpret_cast<float4*>(gs + 4) = *reinterpret_cast<const float4*>(sc + l + 4);
                  *reinterpret_cast<float4*>(us) = *reinterpret_cast<const float4*>(sc + 128 + l);
                  *reinterpret_cast<float4*>(us + 4) = *reinterpret_cast<const float4*>(sc + 128 + l + 4);
                }
                float h[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  float gv = acc_value<KIND>(g[8 * j + i]);
                  float uv = acc_value<KIND>(u[8 * j + i]);
                  if constexpr (KIND == 2) {
                    gv = gv * sa * gs[i];
                    uv = uv * sa * us[i];
                  }
                  h[i] = silu_mul(gv, uv);
                }
                store8_out(p.out, p.out_dtype, grow * p.ldo + cj, h);
              }
            }
          }
          chunk_done(c);
        }
      } else {
        int64_t dst_row = grow;
        const float wgt = cur.wgt;
        bool do_store = row_ok;
        void* obase = p.out;
        if (p.epi != MOE_EPI_STORE_ROWS && row_ok) {
          const int32_t slot = cur.slot;
          do_store = slot >= 0;
          if (slot >= 0) {
            if (p.epi == kEpiScatterPeer) {
              const int src = slot >> 24;
              dst_row = slot & 0xFFFFFF;
              if (src < p.num_peers) obase = p.peer_out[src];
              else do_store = false;
            } else {
              dst_row = (p.epi == MOE_EPI_COMBINE_ADD) ? (int64_t)(slot / p.top_k) : (int64_t)slot;
            }
          }
        }
        if (dst_row >= p.out_rows) do_store = false;
        // whole unit: N tile columns [0, 256) at TMEM columns [0, 256); half
        // unit: this lane's half of the N tile at TMEM columns [0, 128)
        const int ncols = half ? BN / 2 : BN;
        const int lbase = half ? (q >> 1) * (BN / 2) : 0;  // first column of this lane within the N tile
        const int cbase = n * BN + lbase;
        if (p.out_dtype != MOE_F32 && p.epi != MOE_EPI_COMBINE_ADD) {
          uint8_t* stage = epi_stage + (warp - 2) * STAGE_WARP_BYTES;
#pragma unroll 1
          for (int c2 = 0; c2 < ncols / 64; ++c2) {
            uint32_t v0[32], v1[32];
            ptx::tmem_ld32(tbase + c2 * 64, v0);
            ptx::tmem_ld32(tbase + c2 * 64 + 32, v1);
            ptx::tmem_ld_wait();
            const int col0 = cbase + c2 * 64;
            uint32_t packed[32];
#pragma unroll
            for (int i4 = 0; i4 < 16; ++i4) {
              float s4[4] = {1.f, 1.f, 1.f, 1.f};
              if constexpr (KIND == 2)
                *reinterpret_cast<float4*>(s4) = *reinterpret_cast<const float4*>(sc + lbase + c2 * 64 + 4 * i4);
#pragma unroll
              for (int h2 = 0; h2 < 2; ++h2) {
                const int i = 2 * i4 + h2;  // packed pair: columns col0 + 2i, col0 + 2i + 1
                const uint32_t* src = i < 16 ? v0 : v1;
                const int li = (i & 15) * 2;
                float a = acc_value<KIND>(src[li]), b = acc_value<KIND>(src[li + 1]);
                if constexpr (KIND == 2) {
                  a = a * sa * s4[2 * h2];
                  b = b * sa * s4[2 * h2 + 1];
                }
                packed[i] = pack2(a * wgt, b * wgt, p.out_dtype);
              }
            }
            const int nvalid = min(64, p.n_valid - col0);
            const unsigned long long rp =
                (do_store && nvalid > 0) ? reinterpret_cast<unsigned long long>(static_cast<char*>(obase) +
                                                                               (dst_row * p.ldo + col0) * 2)
                                         : 0ull;
            staged_store<8>(stage, packed, rp, nvalid > 0 ? nvalid * 2 : 0, lane);
            chunk_done(c2);
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < ncols / 32; ++c) {
            uint32_t v[32];
            ptx::tmem_ld32(tbase + c * 32, v);
            ptx::tmem_ld_wait();
            const int col0 = cbase + c * 32;
            if (do_store && col0 < p.n_valid) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int cj = col0 + 8 * j;
                if (cj < p.n_valid) {
                  float s8[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
                  if constexpr (KIND == 2) {
                    const int l = lbase + c * 32 + 8 * j;
                    *reinterpret_cast<float4*>(s8) = *reinterpret_cast<const float4*>(sc + l);
                    *reinterpret_cast<float4*>(s8 + 4) = *reinterpret_cast<const float4*>(sc + l + 4);
                  }
                  float f[8];
#pragma unroll
                  for (int i = 0; i < 8; ++i) {
                    float x = acc_value<KIND>(v[8 * j + i]);
                    if constexpr (KIND == 2) x = x * sa * s8[i];
                    f[i] = x * wgt;
                  }
                  if (p.epi == MOE_EPI_COMBINE_ADD) {
                    float* dst = static_cast<float*>(p.out) + dst_row * p.ldo + cj;
                    red_add4(dst, f[0], f[1], f[2], f[3]);
                    red_add4(dst + 4, f[4], f[5], f[6], f[7]);
                  } else {
                    store8_out(obase, p.out_dtype, dst_row * p.ldo + cj, f);
                  }
                }
              }
            }
            chunk_done(c);
          }
        }
      }
      // the next tile's column scales into the other buffer (its loads were
      // issued before this tile drained)
      if (nxt.live) stage_scales(nxt, (it + 1) & 1);
      ptx::tc_fence_before();
      if constexpr (PAIR) ptx::mbar_arrive_cluster(tempty_leader[acc]);
      else ptx::mbar_arrive(&tempty[acc]);
      cur = nxt;
    }
    if (!ok) {
      if (lane == 0) raise_device_error(3);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  clock_end(clk);
  if constexpr (PAIR) ptx::cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    if constexpr (PAIR) ptx::tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Waits on an mbarrier that nothing ever completes: the bounded wait must give
// up after timeout_ns and latch error code 6 (self-test of the timeout path).
__global__ void selftest_wait_kernel(uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !ptx::mbar_wait(&bar, 0, &abort_flag, timeout_ns)) raise_device_error(6);
}

// ---------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode(EncodeTiledFn* fn) {
  struct Entry {
    EncodeTiledFn fn = nullptr;
    cudaError_t err = cudaSuccess;
  };
  static const Entry entry = [] {  // looked up once, thread-safe
    Entry r;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    r.err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (r.err == cudaSuccess && q == cudaDriverEntryPointSuccess) r.fn = reinterpret_cast<EncodeTiledFn>(ptr);
    return r;
  }();
  if (!entry.fn)
    return set_error(MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(entry.err));
  *fn = entry.fn;
  return MOE_OK;
}

int make_tmap(CUtensorMap* m, const void* ptr, int dtype, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn enc;
  MOE_TRY(get_encode(&enc));
  const int es = dtype_size(dtype);
  CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (dtype == MOE_F16) dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  else if (dtype == MOE_F32) dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  else if (dtype == MOE_I8) dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * es};
  cuuint32_t box[2] = {(cuuint32_t)(ROW_BYTES / es), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %llu x %llu dtype %d", (int)r,
                     (unsigned long long)rows, (unsigned long long)inner, dtype);
  return MOE_OK;
}

// tcgen05 instruction descriptor: accumulator format, A/B formats, N, M.
uint32_t make_idesc(int dtype, int m) {
  int c_fmt = 1, ab = 1;  // fp32 accumulate, bf16 operands
  if (dtype == MOE_F16) ab = 0;
  else if (dtype == MOE_F32) ab = 2;  // tf32
  else if (dtype == MOE_I8) {
    c_fmt = 2;  // s32 accumulate
    ab = 1;     // signed int8
  }
  return ((uint32_t)c_fmt << 4) | ((uint32_t)ab << 7) | ((uint32_t)ab << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

int kind_of(int dtype) { return dtype == MOE_F32 ? 1 : (dtype == MOE_I8 ? 2 : 0); }

// GEMM variant: 1 = CTA pairs (cta_group::2), 0 = one CTA per tile,
// 2 = automatic: pairs when the experts average at least 4 M tiles (measured:
// Mixtral layer, 9 tiles per expert, pairs 3 % faster per step), or when the
// launch has fewer (M tile, N tile) units than SMs, where a pair spreads each
// unit's weight stream over two SMs (Qwen3 decode at 1 token: 0.056 vs
// 0.064 ms per step); one CTA per tile otherwise (DeepSeek-V3 w8a8 at one GPU,
// 2 tiles per expert: 3.81 vs 4.28 ms per step; Qwen3 decode at 256 tokens:
// 0.277 vs 0.290 ms).
std::atomic<int> g_gemm_cta_pair{2};
std::atomic<int> g_gemm_band{GROUP_M};  // M tiles per band of the tile raster
std::atomic<int> g_gemm_band_down{0};   // the down GEMM's band (0: g_gemm_band)
// Stream-K split of the partial last wave for the additive combine epilogue.
// Off by default: on the Mixtral layer the down GEMM measured 0.760 ms with it
// and 0.745 ms without (the persistent grid's tail costs less than the extra
// partial-tile epilogues and the K-split tail's weaker L2 reuse).
std::atomic<int> g_gemm_stream_k{0};
// CTA pairs: an expert's odd last M tile as one M=128 pair MMA (64 rows per
// CTA) instead of an M=256 one with one CTA's half idle.
std::atomic<int> g_gemm_half_units{1};
// Programmatic dependent launch for every kernel of the library.
std::atomic<int> g_pdl{1};
// Device-side timing of the GEMM launches (MOE_OPT_KERNEL_CLOCKS).
std::atomic<int> g_kernel_clocks_on{0};
// Swapped operand roles for few rows per expert (MOE_OPT_GEMM_SWAP_AB).
std::atomic<int> g_gemm_swap{2};
// Auto rule: swap when the routed rows average at most this many per expert
// that receives any.
constexpr int64_t kSwapRowsPerExpert = 64;

bool use_pair(int64_t max_tiles, int E, int64_t n_tiles) {
  const int v = g_gemm_cta_pair.load();
  if (v == 2) return max_tiles >= 4 * (int64_t)E || max_tiles * n_tiles < num_sms();
  return v != 0;
}

template <bool PAIR>
size_t gemm_smem_bytes(int E, bool int8_scales) {
  return 1024 + (size_t)Cfg<PAIR>::kStages * Cfg<PAIR>::kStageBytes + BAR_BYTES + align_up16(2 * (E + 1) * 4) +
         EPI_STAGE_BYTES + (int8_scales ? EPI_SCALE_BYTES : 0);
}

template <int KIND, bool SWIGLU, bool PAIR>
int launch_kind(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta64, const CUtensorMap& tb64,
                const Params& p, int64_t units_ub, cudaStream_t st) {
  const size_t smem = gemm_smem_bytes<PAIR>(p.E, KIND == 2);
  auto kfn = moe_gemm_kernel<KIND, SWIGLU, PAIR>;
  MOE_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  int64_t grid;
  if constexpr (PAIR) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * (unsigned)(num_sms() / 2));
    int clusters = 0;
    MOE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kfn, &cfg));
    if (clusters <= 0) return set_error(MOE_ERR_CUDA, "moe_gemm_kernel: no CTA pair fits on the device");
    grid = 2 * std::min<int64_t>(clusters, units_ub);
  } else {
    grid = std::min<int64_t>(num_sms(), units_ub);
  }
  if (grid <= 0) return MOE_OK;
  cfg.gridDim = dim3((unsigned)grid);
  if (pdl_enabled()) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs += 1;
  }
  MOE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, ta, tb, ta64, tb64, p));
  MOE_LAUNCH_CHECK("moe_gemm_kernel");
  return MOE_OK;
}

template <bool SWIGLU, bool PAIR>
int launch(int dtype, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta64, const CUtensorMap& tb64,
           const Params& p, cudaStream_t st) {
  // units: M tiles (single CTA) or M-tile pairs, upper bound max_tiles
  const int64_t units_ub = (int64_t)(PAIR ? (p.max_tiles + p.E) / 2 + p.E : p.max_tiles) * p.n_tiles;
  switch (kind_of(dtype)) {
    case 0: return launch_kind<0, SWIGLU, PAIR>(ta, tb, ta64, tb64, p, units_ub, st);
    case 1: return launch_kind<1, SWIGLU, PAIR>(ta, tb, ta64, tb64, p, units_ub, st);
    default: return launch_kind<2, SWIGLU, PAIR>(ta, tb, ta64, tb64, p, units_ub, st);
  }
}

int check_gemm_common(const char* fn, int dtype, int64_t k, int E, const int32_t* table, int64_t max_tiles) {
  MOE_CHECK_ARG(dtype == MOE_BF16 || dtype == MOE_F16 || dtype == MOE_F32 || dtype == MOE_I8,
                "%s: unsupported dtype %d", fn, dtype);
  const int es = dtype_size(dtype);
  MOE_CHECK_ARG(k > 0 && (k * es) % 16 == 0, "%s: reduction length %lld x %d bytes must be a multiple of 16 bytes",
                fn, (long long)k, es);
  MOE_CHECK_ARG(E > 0 && E <= MAX_GEMM_EXPERTS, "%s: num_experts %d outside [1, %d]", fn, E, MAX_GEMM_EXPERTS);
  MOE_CHECK_ARG(table != nullptr, "%s: tile_table is NULL", fn);
  MOE_CHECK_ARG(max_tiles >= 0 && max_tiles < (int64_t(1) << 24), "%s: max_tiles out of range", fn);
  return MOE_OK;
}

}  // namespace
}  // namespace moe

#include "moe_gemm_swap.cuh"
#include "moe_decode.cuh"

using namespace moe;

extern "C" int moe_get_device_error(int* host_code, void* stream) {
  MOE_CHECK_ARG(host_code != nullptr, "moe_get_device_error: NULL output");
  cudaStream_t st = as_stream(stream);
  int zero = 0;
  MOE_CUDA_TRY(cudaMemcpyFromSymbolAsync(host_code, g_moe_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st));
  MOE_CUDA_TRY(cudaMemcpyToSymbolAsync(g_moe_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st));
  MOE_CUDA_TRY(cudaStreamSynchronize(st));
  if (*host_code != 0) {
    // a failed launch of the one-launch decode kernel may leave its launch
    // counter partial: clear it and move to a fresh generation, so the next
    // launch's tag differs from every count word the failed one left
    unsigned int gen = 0;
    static const unsigned int z = 0;
    MOE_CUDA_TRY(cudaMemcpyFromSymbolAsync(&gen, g_decode_bar_gen, sizeof(gen), 0, cudaMemcpyDeviceToHost, st));
    MOE_CUDA_TRY(cudaStreamSynchronize(st));
    gen += 1;
    MOE_CUDA_TRY(cudaMemcpyToSymbolAsync(g_decode_bar_gen, &gen, sizeof(gen), 0, cudaMemcpyHostToDevice, st));
    MOE_CUDA_TRY(cudaMemcpyToSymbolAsync(g_decode_bar_count, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st));
    MOE_CUDA_TRY(cudaStreamSynchronize(st));
  }
  return MOE_OK;
}

namespace moe {

GemmPlan gemm_plan(int64_t slots, int num_experts, int64_t max_tiles, int64_t hidden, int64_t inter, int dtype,
                   bool combine) {
  GemmPlan p;
  const int opt = g_gemm_swap.load();
  const int64_t nonempty = std::min<int64_t>(num_experts, slots);
  p.swap = opt == 1 || (opt == 2 && slots > 0 && slots <= kSwapRowsPerExpert * nonempty);
  if (!p.swap) return p;
  p.nmax = (slots > 0 && slots <= 32) ? 32 : 128;
  // the swapped down GEMM streams 16 KB of weights per stage next to the token
  // rows and adds its combine one element at a time: measured against the
  // row-major kernel on Qwen3-30B-A3B decode shapes it ties at 8 routed slots
  // and loses from 64 on (T = 8: 30.2 vs 24.5 us; T = 256: 156 vs 71 us), so
  // it runs only for the smallest batches, where it also converts the output
  p.swap2 = opt == 1 || p.nmax == 32;
  const int64_t sms = num_sms();
  const int es = dtype_size(dtype);
  const int64_t nf1 = ceil_div(inter, SW_FEAT), nf2 = ceil_div(hidden, SW_FEAT);
  const int64_t kb1 = ceil_div(hidden * es, ROW_BYTES), kb2 = ceil_div(inter * es, ROW_BYTES);
  // fewer work items than half the SMs: split K so about one wave of items
  // runs, each split keeping at least 4 K blocks
  auto split = [&](int64_t units, int64_t kb) -> int {
    if (units <= 0 || 2 * units > sms) return 1;
    return (int)std::max<int64_t>(1, std::min<int64_t>(sms / units, kb / 4));
  };
  p.splits1 = split(max_tiles * nf1, kb1);
  p.splits2 = (combine && p.swap2) ? split(max_tiles * nf2, kb2) : 1;
  if (p.splits1 > 1) {
    p.partial_bytes = (size_t)max_tiles * nf1 * p.splits1 * 2 * SW_FEAT * p.nmax * 4;
    p.counter_bytes = (size_t)max_tiles * nf1 * 4 * sizeof(int32_t);
  }
  return p;
}

namespace {
// The swapped-operand plan a stand-alone GEMM call runs with: forced by
// MOE_OPT_GEMM_SWAP_AB = 1 only, 128 token rows per item, no K split.
const GemmPlan* standalone_plan(GemmPlan* storage) {
  if (g_gemm_swap.load() != 1) return nullptr;
  storage->swap = storage->swap2 = true;
  return storage;
}
}  // namespace

int gemm1_swiglu_planned(const void* a, int dtype, int64_t a_rows, int64_t hidden, const void* w13, int num_experts,
                         int64_t inter, const float* a_scale, const float* w13_scale, const int32_t* tile_table,
                         int64_t max_tiles, void* h, int h_dtype, const GemmPlan* plan, void* partial,
                         int32_t* counters, cudaStream_t stream) {
  MOE_TRY(check_gemm_common("moe_gemm1_swiglu", dtype, hidden, num_experts, tile_table, max_tiles));
  MOE_CHECK_ARG(a && w13 && h, "moe_gemm1_swiglu: NULL pointer");
  MOE_CHECK_ARG(inter > 0 && inter % 8 == 0, "moe_gemm1_swiglu: inter (%lld) must be a positive multiple of 8",
                (long long)inter);
  MOE_CHECK_ARG(a_rows >= 0 && a_rows < (int64_t(1) << 31), "moe_gemm1_swiglu: a_rows out of range");
  MOE_CHECK_ARG((int64_t)num_experts * 2 * inter < (int64_t(1) << 31), "moe_gemm1_swiglu: weight rows overflow");
  MOE_CHECK_ARG(h_dtype == MOE_BF16 || h_dtype == MOE_F16 || h_dtype == MOE_F32, "moe_gemm1_swiglu: bad h dtype");
  if (dtype == MOE_I8) MOE_CHECK_ARG(a_scale && w13_scale, "moe_gemm1_swiglu: int8 needs a_scale and w13_scale");
  MOE_CHECK_ARG((uintptr_t)a % 16 == 0 && (uintptr_t)w13 % 16 == 0 && (uintptr_t)h % 16 == 0,
                "moe_gemm1_swiglu: pointers must be 16-byte aligned");
  if (a_rows == 0 || max_tiles == 0) return MOE_OK;
  if (plan && plan->swap) {
    const int splits = plan->splits1;
    if (splits > 1) MOE_CHECK_ARG(partial && counters, "moe_gemm1_swiglu: a K split needs its workspace");
    CUtensorMap tw, tx;
    MOE_TRY(make_tmap(&tw, w13, dtype, hidden, (uint64_t)num_experts * 2 * inter, SW_FEAT));
    MOE_TRY(make_tmap(&tx, a, dtype, hidden, a_rows, SW_BOX));
    SwapParams p{};
    p.E = num_experts;
    p.num_kb = (int)ceil_div(hidden * dtype_size(dtype), ROW_BYTES);
    p.splits = splits;
    p.nf = (int)ceil_div(inter, SW_FEAT);
    p.n_valid = (int)inter;
    p.w_rows_per_expert = (int)(2 * inter);
    p.inter = (int)inter;
    p.nmax = plan->nmax;
    p.stages = swap_stages(true, p.nmax, num_experts);
    p.idesc_m = make_idesc(dtype, SW_FEAT) & ~(0x3Fu << 17);
    p.table = tile_table;
    p.max_tiles = (int)max_tiles;
    p.a_rows = a_rows;
    p.epi = MOE_EPI_STORE_ROWS;
    p.out = h;
    p.out_dtype = h_dtype;
    p.ldo = inter;
    p.out_rows = a_rows;
    p.a_scale = a_scale;
    p.w_scale = w13_scale;
    p.top_k = 1;
    p.partial = partial;
    p.counters = counters;
    p.clock_slot = g_kernel_clocks_on.load() ? MOE_CLOCK_GATE_UP : -1;
    return launch_swap<true>(dtype, tw, tx, p, stream);
  }
  CUtensorMap ta, tb, ta64, tb64;
  const bool pair = use_pair(max_tiles, num_experts, ceil_div(inter, BN / 2));
  const bool half_units = pair && g_gemm_half_units.load() != 0;
  MOE_TRY(make_tmap(&ta, a, dtype, hidden, a_rows, BM));
  MOE_TRY(make_tmap(&tb, w13, dtype, hidden, (uint64_t)num_experts * 2 * inter, BN / 2));
  if (half_units) {
    MOE_TRY(make_tmap(&ta64, a, dtype, hidden, a_rows, BM / 2));
    MOE_TRY(make_tmap(&tb64, w13, dtype, hidden, (uint64_t)num_experts * 2 * inter, BN / 4));
  } else {
    ta64 = ta;
    tb64 = tb;
  }
  Params p{};
  p.E = num_experts;
  p.num_kb = (int)ceil_div(hidden * dtype_size(dtype), ROW_BYTES);
  p.n_tiles = (int)ceil_div(inter, BN / 2);
  p.n_valid = (int)inter;
  p.b_rows_per_expert = (int)(2 * inter);
  p.inter = (int)inter;
  p.idesc = make_idesc(dtype, pair ? 2 * BM : BM);
  p.idesc_half = make_idesc(dtype, BM);
  p.half_units = half_units;
  p.band_tiles = g_gemm_band.load();
  p.table = tile_table;
  p.max_tiles = (int)max_tiles;
  p.a_rows = a_rows;
  p.epi = MOE_EPI_STORE_ROWS;
  p.out = h;
  p.out_dtype = h_dtype;
  p.ldo = inter;
  p.out_rows = a_rows;
  p.a_scale = a_scale;
  p.b_scale = w13_scale;
  p.top_k = 1;
  p.clock_slot = g_kernel_clocks_on.load() ? MOE_CLOCK_GATE_UP : -1;
  return pair ? launch<true, true>(dtype, ta, tb, ta64, tb64, p, stream)
              : launch<true, false>(dtype, ta, tb, ta64, tb64, p, stream);
}
}  // namespace moe

extern "C" int moe_gemm1_swiglu(const void* a, int dtype, int64_t a_rows, int64_t hidden, const void* w13,
                                int num_experts, int64_t inter, const float* a_scale, const float* w13_scale,
                                const int32_t* tile_table, int64_t max_tiles, void* h, int h_dtype, void* stream) {
  GemmPlan storage;
  return gemm1_swiglu_planned(a, dtype, a_rows, hidden, w13, num_experts, inter, a_scale, w13_scale, tile_table,
                              max_tiles, h, h_dtype, standalone_plan(&storage), nullptr, nullptr, as_stream(stream));
}

namespace moe {
namespace {
int gemm2_impl(const void* h, int dtype, int64_t h_rows, int64_t inter, const void* w2, int num_experts,
               int64_t hidden, const float* h_scale, const float* w2_scale, const int32_t* tile_table,
               int64_t max_tiles, int epilogue, const int32_t* row_map, const float* row_weight, int top_k,
               void* out, int out_dtype, int64_t out_rows, void* const* peer_out, int num_peers,
               const GemmPlan* plan, cudaStream_t stream, const FusedConvert* convert = nullptr) {
  MOE_TRY(check_gemm_common("moe_gemm2", dtype, inter, num_experts, tile_table, max_tiles));
  MOE_CHECK_ARG(h && w2 && (out || peer_out), "moe_gemm2: NULL pointer");
  MOE_CHECK_ARG(hidden > 0 && hidden % 8 == 0, "moe_gemm2: hidden (%lld) must be a positive multiple of 8",
                (long long)hidden);
  MOE_CHECK_ARG(h_rows >= 0 && h_rows < (int64_t(1) << 31), "moe_gemm2: h_rows out of range");
  MOE_CHECK_ARG((int64_t)num_experts * hidden < (int64_t(1) << 31), "moe_gemm2: weight rows overflow");
  if (epilogue == MOE_EPI_COMBINE_ADD) {
    MOE_CHECK_ARG(out_dtype == MOE_F32, "moe_gemm2: the combine epilogue accumulates into fp32");
    MOE_CHECK_ARG(row_map && row_weight && top_k > 0, "moe_gemm2: combine needs row_map, row_weight, top_k");
  } else {
    MOE_CHECK_ARG(out_dtype == MOE_BF16 || out_dtype == MOE_F16 || out_dtype == MOE_F32, "moe_gemm2: bad out dtype");
  }
  if (epilogue == MOE_EPI_SCATTER_ROWS || epilogue == kEpiScatterPeer)
    MOE_CHECK_ARG(row_map != nullptr, "moe_gemm2: scatter needs row_map");
  if (dtype == MOE_I8) MOE_CHECK_ARG(h_scale && w2_scale, "moe_gemm2: int8 needs h_scale and w2_scale");
  MOE_CHECK_ARG((uintptr_t)h % 16 == 0 && (uintptr_t)w2 % 16 == 0 && (uintptr_t)out % 16 == 0,
                "moe_gemm2: pointers must be 16-byte aligned");
  if (h_rows == 0 || max_tiles == 0) return MOE_OK;
  if (plan && plan->swap2 && epilogue != kEpiScatterPeer) {
    CUtensorMap tw, tx;
    MOE_TRY(make_tmap(&tw, w2, dtype, inter, (uint64_t)num_experts * hidden, SW_FEAT));
    MOE_TRY(make_tmap(&tx, h, dtype, inter, h_rows, SW_BOX));
    SwapParams p{};
    p.E = num_experts;
    p.num_kb = (int)ceil_div(inter * dtype_size(dtype), ROW_BYTES);
    p.splits = epilogue == MOE_EPI_COMBINE_ADD ? plan->splits2 : 1;  // partial sums add only in the combine
    p.nf = (int)ceil_div(hidden, SW_FEAT);
    p.n_valid = (int)hidden;
    p.w_rows_per_expert = (int)hidden;
    p.inter = (int)inter;
    p.nmax = plan->nmax;
    p.stages = swap_stages(false, p.nmax, num_experts);
    p.idesc_m = make_idesc(dtype, SW_FEAT) & ~(0x3Fu << 17);
    p.table = tile_table;
    p.max_tiles = (int)max_tiles;
    p.a_rows = h_rows;
    p.epi = epilogue;
    p.out = out;
    p.out_dtype = out_dtype;
    p.ldo = hidden;
    p.out_rows = out_rows;
    p.a_scale = h_scale;
    p.w_scale = w2_scale;
    p.row_map = row_map;
    p.row_weight = row_weight;
    p.top_k = top_k > 0 ? top_k : 1;
    p.clock_slot = g_kernel_clocks_on.load() ? MOE_CLOCK_DOWN : -1;
    if (convert && epilogue == MOE_EPI_COMBINE_ADD) {
      MOE_CHECK_ARG(convert->out && convert->counters && convert->kvalid, "moe_gemm2: incomplete fused conversion");
      p.conv_out = convert->out;
      p.conv_dtype = convert->dtype;
      p.conv_cnt = convert->counters;
      p.conv_kvalid = convert->kvalid;
    }
    return launch_swap<false>(dtype, tw, tx, p, stream);
  }
  CUtensorMap ta, tb, ta64;
  const bool pair = use_pair(max_tiles, num_experts, ceil_div(hidden, BN));
  const bool half_units = pair && g_gemm_half_units.load() != 0;  // read once: the maps must match
  MOE_TRY(make_tmap(&ta, h, dtype, inter, h_rows, BM));
  if (half_units) MOE_TRY(make_tmap(&ta64, h, dtype, inter, h_rows, BM / 2));
  else ta64 = ta;
  MOE_TRY(make_tmap(&tb, w2, dtype, inter, (uint64_t)num_experts * hidden, pair ? BN / 2 : BN));
  Params p{};
  p.E = num_experts;
  p.num_kb = (int)ceil_div(inter * dtype_size(dtype), ROW_BYTES);
  p.n_tiles = (int)ceil_div(hidden, BN);
  p.n_valid = (int)hidden;
  p.b_rows_per_expert = (int)hidden;
  p.inter = (int)inter;
  p.idesc = make_idesc(dtype, pair ? 2 * BM : BM);
  p.idesc_half = make_idesc(dtype, BM);
  p.half_units = half_units;
  p.band_tiles = g_gemm_band_down.load() ? g_gemm_band_down.load() : g_gemm_band.load();
  p.table = tile_table;
  p.max_tiles = (int)max_tiles;
  p.a_rows = h_rows;
  p.epi = epilogue;
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldo = hidden;
  p.out_rows = out_rows;
  p.a_scale = h_scale;
  p.b_scale = w2_scale;
  p.row_map = row_map;
  p.row_weight = row_weight;
  p.top_k = top_k > 0 ? top_k : 1;
  p.peer_out = peer_out;
  p.num_peers = num_peers;
  // the weighted combine adds partial sums, so its work can be split along K
  // evenly over the grid (no partly idle last wave)
  p.stream_k = epilogue == MOE_EPI_COMBINE_ADD && g_gemm_stream_k.load() != 0;
  p.clock_slot = g_kernel_clocks_on.load() ? MOE_CLOCK_DOWN : -1;
  return pair ? launch<false, true>(dtype, ta, tb, ta64, tb, p, stream)
              : launch<false, false>(dtype, ta, tb, ta64, tb, p, stream);
}
}  // namespace

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

int gemm2_scatter_peer(const void* h, int dtype, int64_t h_rows, int64_t inter, const void* w2, int num_experts,
                       int64_t hidden, const float* h_scale, const float* w2_scale, const int32_t* tile_table,
                       int64_t max_tiles, const int32_t* row_meta, void* const* peer_out, int num_peers,
                       int64_t peer_rows, int out_dtype, cudaStream_t stream) {
  MOE_CHECK_ARG(peer_out && num_peers > 0 && num_peers <= 256, "ep: bad peer output table");
  return gemm2_impl(h, dtype, h_rows, inter, w2, num_experts, hidden, h_scale, w2_scale, tile_table, max_tiles,
                    kEpiScatterPeer, row_meta, nullptr, 1, nullptr, out_dtype, peer_rows, peer_out, num_peers,
                    nullptr, stream);
}

int gemm2_planned(const void* h, int dtype, int64_t h_rows, int64_t inter, const void* w2, int num_experts,
                  int64_t hidden, const float* h_scale, const float* w2_scale, const int32_t* tile_table,
                  int64_t max_tiles, int epilogue, const int32_t* row_map, const float* row_weight, int top_k,
                  void* out, int out_dtype, int64_t out_rows, const GemmPlan* plan, cudaStream_t stream,
                  const FusedConvert* convert) {
  MOE_CHECK_ARG(out != nullptr, "moe_gemm2: NULL pointer");
  return gemm2_impl(h, dtype, h_rows, inter, w2, num_experts, hidden, h_scale, w2_scale, tile_table, max_tiles,
                    epilogue, row_map, row_weight, top_k, out, out_dtype, out_rows, nullptr, 0, plan, stream,
                    convert);
}
}  // namespace moe

extern "C" int moe_gemm2(const void* h, int dtype, int64_t h_rows, int64_t inter, const void* w2, int num_experts,
                         int64_t hidden, const float* h_scale, const float* w2_scale, const int32_t* tile_table,
                         int64_t max_tiles, int epilogue, const int32_t* row_map, const float* row_weight,
                         int top_k, void* out, int out_dtype, int64_t out_rows, void* stream) {
  MOE_CHECK_ARG(epilogue == MOE_EPI_STORE_ROWS || epilogue == MOE_EPI_COMBINE_ADD || epilogue == MOE_EPI_SCATTER_ROWS,
                "moe_gemm2: bad epilogue %d", epilogue);
  MOE_CHECK_ARG(out != nullptr, "moe_gemm2: NULL pointer");
  GemmPlan storage;
  return gemm2_impl(h, dtype, h_rows, inter, w2, num_experts, hidden, h_scale, w2_scale, tile_table, max_tiles,
                    epilogue, row_map, row_weight, top_k, out, out_dtype, out_rows, nullptr, 0,
                    standalone_plan(&storage), as_stream(stream));
}

extern "C" int moe_set_option(int option, int value) {
  if (option == MOE_OPT_GEMM_CTA_PAIR) {
    MOE_CHECK_ARG(value >= 0 && value <= 2, "moe_set_option: GEMM_CTA_PAIR takes 0, 1 or 2");
    g_gemm_cta_pair.store(value);
    return MOE_OK;
  }
  if (option == MOE_OPT_GEMM_BAND) {
    MOE_CHECK_ARG(value >= 1 && value <= 1 << 20, "moe_set_option: GEMM_BAND takes 1 .. 2^20 tiles");
    g_gemm_band.store(value);
    return MOE_OK;
  }
  if (option == MOE_OPT_DECODE_FUSED) {
    MOE_CHECK_ARG(value >= 0 && value <= 2, "moe_set_option: DECODE_FUSED takes 0, 1 or 2");
    g_decode_fused.store(value);
    return MOE_OK;
  }
  if (option == MOE_OPT_GEMM_BAND_DOWN) {
    MOE_CHECK_ARG(value >= 0 && value <= 1 << 20, "moe_set_option: GEMM_BAND_DOWN takes 0 .. 2^20 tiles");
    g_gemm_band_down.store(value);
    return MOE_OK;
  }
  if (option == MOE_OPT_GEMM_STREAM_K) {
    g_gemm_stream_k.store(value != 0);
    return MOE_OK;
  }
  if (option == MOE_OPT_GEMM_HALF_UNITS) {
    g_gemm_half_units.store(value != 0);
    return MOE_OK;
  }
  if (option == MOE_OPT_PDL) {
    g_pdl.store(value != 0);
    return MOE_OK;
  }
  if (option == MOE_OPT_KERNEL_CLOCKS) {
    g_kernel_clocks_on.store(value != 0);
    return MOE_OK;
  }
  if (option == MOE_OPT_GEMM_SWAP_AB) {
    MOE_CHECK_ARG(value >= 0 && value <= 2, "moe_set_option: GEMM_SWAP_AB takes 0, 1 or 2");
    g_gemm_swap.store(value);
    return MOE_OK;
  }
  return set_error(MOE_ERR_INVALID_ARG, "moe_set_option: unknown option %d", option);
}

extern "C" int moe_get_option(int option) {
  if (option == MOE_OPT_GEMM_CTA_PAIR) return g_gemm_cta_pair.load();
  if (option == MOE_OPT_GEMM_BAND) return g_gemm_band.load();
  if (option == MOE_OPT_GEMM_BAND_DOWN) return g_gemm_band_down.load();
  if (option == MOE_OPT_DECODE_FUSED) return g_decode_fused.load();
  if (option == MOE_OPT_GEMM_STREAM_K) return g_gemm_stream_k.load();
  if (option == MOE_OPT_GEMM_HALF_UNITS) return g_gemm_half_units.load();
  if (option == MOE_OPT_PDL) return g_pdl.load();
  if (option == MOE_OPT_KERNEL_CLOCKS) return g_kernel_clocks_on.load();
  if (option == MOE_OPT_GEMM_SWAP_AB) return g_gemm_swap.load();
  return -1;
}

extern "C" int moe_kernel_clocks(uint64_t* total_ns, uint64_t* launches, int n, int reset, void* stream) {
  MOE_CHECK_ARG(n >= 0 && n <= MOE_NUM_CLOCKS, "moe_kernel_clocks: n must be in [0, %d]", MOE_NUM_CLOCKS);
  MOE_CHECK_ARG(n == 0 || (total_ns && launches), "moe_kernel_clocks: NULL output");
  cudaStream_t st = as_stream(stream);
  KernelClock host[MOE_NUM_CLOCKS];
  MOE_CUDA_TRY(cudaMemcpyFromSymbolAsync(host, g_kernel_clocks, sizeof(host), 0, cudaMemcpyDeviceToHost, st));
  if (reset) {
    static const KernelClock zero[MOE_NUM_CLOCKS] = {};
    MOE_CUDA_TRY(cudaMemcpyToSymbolAsync(g_kernel_clocks, zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st));
  }
  MOE_CUDA_TRY(cudaStreamSynchronize(st));
  for (int i = 0; i < n; ++i) {
    total_ns[i] = host[i].total_ns;
    launches[i] = host[i].launches;
  }
  return MOE_OK;
}

extern "C" int moe_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
  MOE_CHECK_ARG(timeout_ns > 0 && timeout_ns <= 2000000000ull, "moe_selftest_wait_timeout: limit must be in (0, 2 s]");
  selftest_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(timeout_ns);
  MOE_LAUNCH_CHECK("selftest_wait_kernel");
  return MOE_OK;
}
