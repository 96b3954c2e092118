// Grouped MoE GEMMs for few rows per expert (decode), operands swapped.
//
// Included by moe_gemm.cu (same translation unit: it shares the device error
// flag, the kernel clocks, the tensor-map helpers and the PTX wrappers).
//
// When an expert receives a handful of token rows, the row-major kernel's
// 128-row M tile is almost all padding, and every pipeline stage ships a
// 128-row activation box next to the weight rows. Here the roles swap: the
// MMA's M=128 operand is 128 weight rows (output features) and its N operand
// is the expert's token rows, N = the rows rounded up to 16, loaded as 16-row
// TMA boxes. The ring then carries weight bytes plus only the real token rows,
// and the accumulator D[feature][token] sits in TMEM with one feature per lane
// and one token per column.
//
// Work item = (M tile of the tile table = one expert's <= 128 token rows,
// feature tile of 128 weight rows, K split). Items run expert-major with the
// token tiles of one (feature tile, split) adjacent, so concurrently running
// CTAs share weight tiles in L2. The gate_up GEMM issues two MMAs per K step
// (128 gate rows and the matching 128 up rows into two accumulators), so one
// thread holds the gate and up values of its feature for SwiGLU.
//
// K splits (launches with fewer (tile, feature tile) units than half the
// SMs): each split accumulates a contiguous share of K. Down GEMM with the
// combine epilogue: the partial sums are added into the fp32 output like any
// other contribution. Gate_up GEMM: each split stores its partial
// accumulators (fp32, or int32 for int8) to a workspace slot; the last split
// to finish a unit (an atomic count per epilogue warp) adds all the unit's
// slots in split order — a fixed order, so results do not depend on which
// split finishes last — and applies SwiGLU.
namespace moe {
namespace {

constexpr int SW_FEAT = 128;            // weight rows per MMA (UMMA M)
constexpr int SW_BOX = 16;              // token rows per TMA box
constexpr int SW_MAX_STAGES = 12;
constexpr int SW_SMEM_BUDGET = 226 * 1024;  // of the 227 KB a CTA may use
constexpr uint32_t SW_A_TILE = SW_FEAT * ROW_BYTES;  // 16 KiB

struct SwapParams {
  int E;
  int num_kb;            // K blocks of 128 bytes
  int splits;             // K splits: split s covers K blocks [s * num_kb / splits, (s + 1) * num_kb / splits)
  int nf;                // feature tiles of 128 rows
  int n_valid;           // valid output features (I for gate_up, H for down)
  int w_rows_per_expert; // weight rows per expert (2I or H)
  int inter;             // gate_up: row offset of the up half within an expert
  int nmax;              // token rows reserved per stage (32 or 128)
  int stages;
  uint32_t idesc_m;      // instruction descriptor without the N field
  const int32_t* table;
  int max_tiles;
  int64_t a_rows;        // rows of the token operand
  int epi;
  void* out;
  int out_dtype;
  int64_t ldo;
  int64_t out_rows;
  const float* a_scale;  // per token row (int8)
  const float* w_scale;  // per weight row (int8)
  const int32_t* row_map;
  const float* row_weight;
  int top_k;
  void* partial;         // gate_up with splits > 1: [units][splits][2][128][nmax] 32-bit
  int32_t* counters;     // gate_up with splits > 1: [units][4], zero on entry, left zero
  int clock_slot;
  // down GEMM, combine epilogue: fused conversion of the fp32 accumulator
  // (out) to conv_out, per (token, 32-feature group), by the warp whose add
  // completes the group: conv_cnt [T][nf * 4] zero on entry, conv_kvalid [T]
  void* conv_out;
  int conv_dtype;
  int32_t* conv_cnt;
  const int32_t* conv_kvalid;
};

__host__ __device__ constexpr int swap_na(bool swiglu) { return swiglu ? 2 : 1; }

// First K block of split s (balanced: every split is non-empty while
// splits <= num_kb).
__device__ __forceinline__ int split_begin(int s, const SwapParams& p) {
  return (int)((int64_t)s * p.num_kb / p.splits);
}

__device__ __forceinline__ void store1_out(void* base, int dtype, int64_t idx, float v) {
  if (dtype == MOE_BF16) static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  else if (dtype == MOE_F16) static_cast<__half*>(base)[idx] = __float2half_rn(v);
  else static_cast<float*>(base)[idx] = v;
}

__device__ __forceinline__ void red_add1(float* addr, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}

// item -> (expert e, M tile m, feature tile f, split s); expert-major, then
// feature tile, then split, then the expert's token tiles.
__device__ __forceinline__ void swap_decode(int item, const int32_t* s_cum, int E, int nf, int splits, int& e, int& m,
                                            int& f, int& s) {
  const int per = nf * splits;
  int lo = 0, hi = E;  // s_cum[lo] * per <= item < s_cum[hi] * per
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s_cum[mid] * per <= item) lo = mid;
    else hi = mid;
  }
  e = lo;
  const int tiles = s_cum[e + 1] - s_cum[e];
  const int local = item - s_cum[e] * per;
  m = s_cum[e] + local % tiles;
  const int rest = local / tiles;
  s = rest % splits;
  f = rest / splits;
}

template <int KIND, bool SWIGLU>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    moe_gemm_swap_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                         const SwapParams p) {
  constexpr int NA = swap_na(SWIGLU);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  const uint32_t b_bytes = (uint32_t)p.nmax * ROW_BYTES;
  const uint32_t stage_bytes = NA * SW_A_TILE + b_bytes;
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + SW_MAX_STAGES;
  uint64_t* tfull = empty + SW_MAX_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_cum = reinterpret_cast<int32_t*>(smem + (size_t)S * stage_bytes + BAR_BYTES);
  // per epilogue warp: the current item's token slots, routing weights and
  // activation scales (staged once per item, read back as broadcasts)
  int32_t* s_meta = s_cum + align_up16((p.E + 1) * 4) / 4;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const uint32_t tmem_cols = SWIGLU ? (p.nmax == 128 ? 512u : 128u) : (p.nmax == 128 ? 256u : 64u);
  const int acc_stride = NA * p.nmax;  // TMEM columns per accumulator buffer

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      ptx::mbar_init(&full[i], 1);
      ptx::mbar_init(&empty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      ptx::mbar_init(&tempty[a], 4 * 32);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_w);
    ptx::prefetch_tmap(&tmap_x);
  }
  pdl_begin();
  KernelClock* const clk = p.clock_slot >= 0 ? &g_kernel_clocks[p.clock_slot] : nullptr;
  clock_begin(clk);
  for (int i = threadIdx.x; i <= E; i += blockDim.x) s_cum[i] = p.table[TileTable::cum_off() + i];
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, tmem_cols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = s_cum[E] * p.nf * p.splits;
  const int32_t* row_start_tab = p.table + TileTable::start_off(E);
  const int32_t* row_count_tab = p.table + TileTable::count_off(E, p.max_tiles);
  constexpr int kElems = ROW_BYTES / (KIND == 0 ? 2 : (KIND == 1 ? 4 : 1));

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_par[SW_MAX_STAGES];
      for (int i = 0; i < SW_MAX_STAGES; ++i) last_par[i] = -1;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x) {
        int e, m, f, s;
        swap_decode(item, s_cum, E, p.nf, p.splits, e, m, f, s);
        const int rstart = row_start_tab[m];
        const int nbox = (row_count_tab[m] + SW_BOX - 1) / SW_BOX;
        const int kb0 = split_begin(s, p), kb1 = split_begin(s + 1, p);
        const int wrow = e * p.w_rows_per_expert + f * SW_FEAT;
        const uint32_t tx = NA * SW_A_TILE + (uint32_t)nbox * SW_BOX * ROW_BYTES;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + (size_t)stage * stage_bytes;
          const int kx = kb * kElems;
          ptx::mbar_arrive_expect_tx(&full[stage], tx);
          ptx::tma_load_2d(st, &tmap_w, &full[stage], kx, wrow);
          if constexpr (SWIGLU) ptx::tma_load_2d(st + SW_A_TILE, &tmap_w, &full[stage], kx, wrow + p.inter);
          for (int b = 0; b < nbox; ++b)
            ptx::tma_load_2d(st + NA * SW_A_TILE + b * SW_BOX * ROW_BYTES, &tmap_x, &full[stage], kx,
                             rstart + b * SW_BOX);
          last_par[stage] = (int)phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        raise_device_error(1);
        *abort_flag = 1;
        volatile int never = 0;
        for (int i = 0; i < S; ++i)
          if (last_par[i] >= 0) ptx::mbar_wait(&full[i], (uint32_t)last_par[i], &never);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int item = blockIdx.x; item < total; item += gridDim.x, ++it) {
        int e, m, f, s;
        swap_decode(item, s_cum, E, p.nf, p.splits, e, m, f, s);
        const int buf = it & 1;
        if (!ptx::mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const int n_mma = (row_count_tab[m] + SW_BOX - 1) / SW_BOX * SW_BOX;
        const uint32_t idesc = p.idesc_m | ((uint32_t)(n_mma >> 3) << 17);
        const uint32_t d = tmem_base + (uint32_t)(buf * acc_stride);
        const int kb0 = split_begin(s, p), kb1 = split_begin(s + 1, p);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(ring + (size_t)stage * stage_bytes);
          const uint32_t b_addr = a_addr + NA * SW_A_TILE;
#pragma unroll
          for (int k = 0; k < ROW_BYTES / 32; ++k) {
            const uint64_t bd = ptx::smem_desc_k128(b_addr + k * 32);
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            ptx::umma<KIND>(d, ptx::smem_desc_k128(a_addr + k * 32), bd, idesc, accum);
            if constexpr (SWIGLU)
              ptx::umma<KIND>(d + p.nmax, ptx::smem_desc_k128(a_addr + SW_A_TILE + k * 32), bd, idesc, accum);
          }
          ptx::umma_commit(&empty[stage]);
          if (++stage == S) {
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
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    bool ok = true;
    int it = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++it) {
      int e, m, f, s;
      swap_decode(item, s_cum, E, p.nf, p.splits, e, m, f, s);
      const int buf = it & 1;
      const bool w_ok = ptx::mbar_wait(&tfull[buf], (it >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const int rstart = row_start_tab[m];
      const int rcount = row_count_tab[m];
      const int fit = q * 32 + lane;            // feature within the tile
      const int feat = f * SW_FEAT + fit;
      const bool feat_ok = feat < p.n_valid;
      const int64_t wrow = (int64_t)e * p.w_rows_per_expert + feat;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * acc_stride);
      const int nchunks = (rcount + 15) / 16;
      float ws_g = 1.f, ws_u = 1.f;
      if constexpr (KIND == 2) {
        ws_g = feat_ok ? p.w_scale[wrow] : 0.f;
        if constexpr (SWIGLU) ws_u = feat_ok ? p.w_scale[wrow + p.inter] : 0.f;
      }
      if (SWIGLU && p.splits > 1) {
        // partial accumulators of this split -> workspace slot, then the last
        // split of the unit sums the slots in split order and applies SwiGLU
        const int unit = m * p.nf + f;
        uint32_t* slot0 = static_cast<uint32_t*>(p.partial) + (size_t)unit * p.splits * 2 * SW_FEAT * p.nmax;
        const size_t split_stride = (size_t)2 * SW_FEAT * p.nmax;
        uint32_t* mine = slot0 + s * split_stride + (size_t)fit * p.nmax;
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
          uint32_t g[16], u[16];
          ptx::tmem_ld16(tbase + c * 16, g);
          ptx::tmem_ld16(tbase + p.nmax + c * 16, u);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            *reinterpret_cast<uint4*>(mine + c * 16 + j) = make_uint4(g[j], g[j + 1], g[j + 2], g[j + 3]);
            *reinterpret_cast<uint4*>(mine + (size_t)SW_FEAT * p.nmax + c * 16 + j) =
                make_uint4(u[j], u[j + 1], u[j + 2], u[j + 3]);
          }
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(&tempty[buf]);
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&p.counters[unit * 4 + q], 1) == p.splits - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          for (int tok = 0; tok < rcount; ++tok) {
            if (!feat_ok) break;
            const int64_t row = (int64_t)rstart + tok;
            float gv, uv;
            if constexpr (KIND == 2) {
              int32_t gi = 0, ui = 0;
              for (int ss = 0; ss < p.splits; ++ss) {
                const uint32_t* src = slot0 + ss * split_stride + (size_t)fit * p.nmax + tok;
                gi += (int32_t)__ldcg(src);
                ui += (int32_t)__ldcg(src + (size_t)SW_FEAT * p.nmax);
              }
              const float sa = p.a_scale[row];
              gv = (float)gi * sa * ws_g;
              uv = (float)ui * sa * ws_u;
            } else {
              gv = 0.f;
              uv = 0.f;
              for (int ss = 0; ss < p.splits; ++ss) {
                const uint32_t* src = slot0 + ss * split_stride + (size_t)fit * p.nmax + tok;
                gv += __uint_as_float(__ldcg(src));
                uv += __uint_as_float(__ldcg(src + (size_t)SW_FEAT * p.nmax));
              }
            }
            store1_out(p.out, p.out_dtype, row * p.ldo + feat, silu_mul(gv, uv));
          }
          __syncwarp();
          if (lane == 0) p.counters[unit * 4 + q] = 0;  // re-armed for the next launch
        }
        continue;
      }
      int32_t* m_slot = s_meta + (warp - 2) * 3 * SW_FEAT;
      float* m_w = reinterpret_cast<float*>(m_slot + SW_FEAT);
      float* m_sa = m_w + SW_FEAT;
      const bool need_slot = !SWIGLU && p.epi != MOE_EPI_STORE_ROWS;
      if (KIND == 2 || need_slot) {
        __syncwarp();  // the previous item's reads of the staging area are done
        for (int tok = lane; tok < rcount; tok += 32) {
          const int64_t row = (int64_t)rstart + tok;
          if constexpr (KIND == 2) m_sa[tok] = p.a_scale[row];
          if (need_slot) {
            const int32_t slot = p.row_map[row];
            m_slot[tok] = slot;
            m_w[tok] = (slot >= 0 && p.row_weight) ? p.row_weight[slot] : 1.f;
          }
        }
        __syncwarp();
      }
#pragma unroll 1
      for (int c = 0; c < nchunks; ++c) {
        uint32_t g[16], u[16];
        ptx::tmem_ld16(tbase + c * 16, g);
        if constexpr (SWIGLU) ptx::tmem_ld16(tbase + p.nmax + c * 16, u);
        ptx::tmem_ld_wait();
        if (!feat_ok) continue;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int tok = c * 16 + j;
          if (tok >= rcount) break;
          const int64_t row = (int64_t)rstart + tok;
          const float sa = KIND == 2 ? m_sa[tok] : 1.f;
          if constexpr (SWIGLU) {
            const float gv = acc_value<KIND>(g[j]) * sa * ws_g;
            const float uv = acc_value<KIND>(u[j]) * sa * ws_u;
            store1_out(p.out, p.out_dtype, row * p.ldo + feat, silu_mul(gv, uv));
          } else {
            const float v = acc_value<KIND>(g[j]) * sa * ws_g;
            if (p.epi == MOE_EPI_STORE_ROWS) {
              if (row < p.out_rows) store1_out(p.out, p.out_dtype, row * p.ldo + feat, v);
            } else {
              const int32_t slot = m_slot[tok];
              if (slot < 0) continue;
              if (p.epi == MOE_EPI_COMBINE_ADD) {
                const int64_t t = slot / p.top_k;
                if (t < p.out_rows) red_add1(static_cast<float*>(p.out) + t * p.ldo + feat, v * m_w[tok]);
              } else if (slot < p.out_rows) {  // MOE_EPI_SCATTER_ROWS
                store1_out(p.out, p.out_dtype, (int64_t)slot * p.ldo + feat, v * m_w[tok]);
              }
            }
          }
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&tempty[buf]);
      if (!SWIGLU && p.conv_out != nullptr) {
        // this warp's adds for its 32 features of the item's tokens are done:
        // count them per token; the warp completing a (token, group) converts it
        __threadfence();
        __syncwarp();
        const int ngroups = p.nf * 4;
        const int group = f * 4 + q;
        for (int t0 = 0; t0 < rcount; t0 += 32) {
          const int tok = t0 + lane;
          int64_t t = -1;
          bool done = false;
          if (tok < rcount) {
            const int32_t slot = p.row_map[(int64_t)rstart + tok];
            if (slot >= 0 && slot / p.top_k < p.out_rows) {
              t = slot / p.top_k;
              const int old = atomicAdd(&p.conv_cnt[t * ngroups + group], 1);
              done = old == p.conv_kvalid[t] * p.splits - 1;
            }
          }
          unsigned todo = __ballot_sync(0xffffffffu, done);
          if (todo) __threadfence();
          while (todo) {
            const int j = __ffs(todo) - 1;
            todo &= todo - 1;
            const int64_t tt = __shfl_sync(0xffffffffu, t, j);
            if (feat_ok)
              store1_out(p.conv_out, p.conv_dtype, tt * p.ldo + feat,
                         __ldcg(static_cast<const float*>(p.out) + tt * p.ldo + feat));
          }
        }
      }
    }
    if (!ok) {
      if (lane == 0) raise_device_error(3);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  clock_end(clk);
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, tmem_cols);
  }
}

// ---------------------------------------------------------------- host side

constexpr size_t SW_META_BYTES = 4 * 3 * SW_FEAT * 4;  // epilogue warps' token metadata staging

size_t swap_smem_bytes(bool swiglu, int nmax, int stages, int E) {
  return 1024 + (size_t)stages * (swap_na(swiglu) * SW_A_TILE + (size_t)nmax * ROW_BYTES) + BAR_BYTES +
         align_up16((E + 1) * 4) + SW_META_BYTES;
}

int swap_stages(bool swiglu, int nmax, int E) {
  const size_t stage = swap_na(swiglu) * SW_A_TILE + (size_t)nmax * ROW_BYTES;
  const size_t fixed = 1024 + BAR_BYTES + align_up16((E + 1) * 4) + SW_META_BYTES;
  return (int)std::min<size_t>(SW_MAX_STAGES, (SW_SMEM_BUDGET - fixed) / stage);
}

template <int KIND, bool SWIGLU>
int launch_swap_kind(const CUtensorMap& tw, const CUtensorMap& tx, const SwapParams& p, int64_t items_ub,
                     cudaStream_t st) {
  const size_t smem = swap_smem_bytes(SWIGLU, p.nmax, p.stages, p.E);
  auto kfn = moe_gemm_swap_kernel<KIND, SWIGLU>;
  MOE_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t grid = std::min<int64_t>(num_sms(), items_ub);
  if (grid <= 0) return MOE_OK;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  MOE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, tw, tx, p));
  MOE_LAUNCH_CHECK("moe_gemm_swap_kernel");
  return MOE_OK;
}

template <bool SWIGLU>
int launch_swap(int dtype, const CUtensorMap& tw, const CUtensorMap& tx, const SwapParams& p, cudaStream_t st) {
  const int64_t items_ub = (int64_t)p.max_tiles * p.nf * p.splits;
  switch (kind_of(dtype)) {
    case 0: return launch_swap_kind<0, SWIGLU>(tw, tx, p, items_ub, st);
    case 1: return launch_swap_kind<1, SWIGLU>(tw, tx, p, items_ub, st);
    default: return launch_swap_kind<2, SWIGLU>(tw, tx, p, items_ub, st);
  }
}

}  // namespace
}  // namespace moe
