// Dense attention for the "flat" query blocks (the reference's
// flash_attn_func call, editing_sparse_attention.py:211-215, fused with the
// scatter and residual of :217-232).
//
// Per CTA: two 128-row query tiles (four 64-token blocks of the flat list)
// share every K/V tile, which halves the L2 -> SM traffic per FLOP.  Roles:
//   warps 0-3  softmax of tile 0 (thread t <-> row t <-> TMEM lane t)
//   warps 4-7  softmax of tile 1 (same lanes, other TMEM columns)
//   warp  8    TMA producer: Q once, then 128-row K and V tiles in two rings
//   warp  9    TMEM allocator and tcgen05.mma issuer
//   warps 10-11 idle (they complete the third warpgroup, which setmaxnreg needs)
// TMEM columns: tile t uses S at [256t, 256t+128) and O at [256t+128, 256t+256).
// After a softmax warpgroup has read S it writes P (bf16 pairs) over the first
// 64 columns of the same region; P.V then reads A from TMEM.  The MMA issue
// order ping-pongs between the tiles:
//   S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) | ...
// so the tensor core works on one tile while the other tile's softmax runs.
// tcgen05.mma instructions of one thread execute in issue order, so S(j+1)
// cannot overwrite P(j) before PV(j) has read it.
#include "icsa_attn_common.cuh"

#include <utility>

namespace icsa {

namespace {

using namespace attn;

constexpr int kFThreads = 384;  // three complete warpgroups (setmaxnreg acts per warpgroup)
constexpr int kFProducerWarp = 8;
constexpr int kFMmaWarp = 9;
constexpr uint32_t kFTmemCols = 512;

template <int D>
struct FCfg {
  static constexpr int kOpBytes = 128 * D * 2;
  static constexpr int kChunks = D / 64;
  static constexpr int kKStages = (D == 128) ? 3 : 4;
  static constexpr int kVStages = (D == 128) ? 2 : 4;
};

template <int D>
struct __align__(1024) FSmem {
  uint8_t q[2][FCfg<D>::kOpBytes];
  uint8_t k[FCfg<D>::kKStages][FCfg<D>::kOpBytes];
  uint8_t v[FCfg<D>::kVStages][FCfg<D>::kOpBytes];
  uint64_t q_full;
  uint64_t k_full[FCfg<D>::kKStages], k_empty[FCfg<D>::kKStages];
  uint64_t v_full[FCfg<D>::kVStages], v_empty[FCfg<D>::kVStages];
  uint64_t s_full[2], p_full[2], o_done[2];
  uint64_t mma_fin;
  uint32_t tmem_base;
  int abort_flag;
};

static_assert(sizeof(FSmem<128>) + 1024 <= 232448, "flat kernel shared memory exceeds 227 KB");
static_assert(sizeof(FSmem<64>) + 1024 <= 232448, "flat kernel shared memory exceeds 227 KB");

struct FTile {
  int bh, b, h;
  int blk[4];    // query blocks of rows [0,64), [64,128) of tile 0 and of tile 1
  int write[4];  // 0 for a duplicate filling an incomplete group
  int n_steps;   // KV steps of 128 rows
};

ICSA_DEV FTile decode_flat_tile(const AttnParams& p, int cta) {
  FTile t;
  const int groups = (p.num_flat + 3) / 4;
  t.bh = cta / groups;
  const int g = cta % groups;
  t.b = t.bh / p.H;
  t.h = t.bh % p.H;
  // flat blocks come first; no order table: query block r is block r
  const int* order = p.order ? p.order + size_t(t.bh) * p.NB : nullptr;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * g + i;
    t.write[i] = r < p.num_flat;
    const int rr = t.write[i] ? r : p.num_flat - 1;
    t.blk[i] = order ? order[rr] : rr;
  }
  t.n_steps = (p.nkv + 1) / 2;
  return t;
}

template <int D>
ICSA_DEV void flat_producer(const AttnParams& p, const AttnMaps& maps, const FTile& t, FSmem<D>& sm) {
  using C = FCfg<D>;
  volatile int* abort_flag = &sm.abort_flag;
  mbar_arrive_expect_tx(&sm.q_full, 2 * C::kOpBytes);
#pragma unroll
  for (int tile = 0; tile < 2; ++tile)
    for (int c = 0; c < C::kChunks; ++c)
      for (int half = 0; half < 2; ++half)
        tma_load_4d(sm.q[tile] + c * kChunkBytes + half * (kChunkBytes / 2), &maps.q, &sm.q_full, c * 64, t.h,
                    t.blk[2 * tile + half] * kBlock, t.b);
  // no block table: KV block i starts at row 64 i
  const int* rows = p.kv_rows ? p.kv_rows + size_t(t.bh) * p.nkv : nullptr;
  for (int j = 0; j < t.n_steps; ++j) {
    const int r0 = rows ? rows[2 * j] : 2 * j * kBlock;
    const int r1 = (2 * j + 1 < p.nkv) ? (rows ? rows[2 * j + 1] : (2 * j + 1) * kBlock) : r0;  // missing half: masked by the softmax
    const int ks = j % C::kKStages;
    if (!mbar_wait(&sm.k_empty[ks], (uint32_t(j / C::kKStages) & 1u) ^ 1u, p.err, kErrKEmpty, abort_flag)) return;
    mbar_arrive_expect_tx(&sm.k_full[ks], C::kOpBytes);
    for (int c = 0; c < C::kChunks; ++c) {
      uint8_t* dst = sm.k[ks] + c * kChunkBytes;
      tma_load_4d(dst, &maps.k, &sm.k_full[ks], c * 64, t.h, r0, t.b);
      tma_load_4d(dst + kChunkBytes / 2, &maps.k, &sm.k_full[ks], c * 64, t.h, r1, t.b);
    }
    const int vs = j % C::kVStages;
    if (!mbar_wait(&sm.v_empty[vs], (uint32_t(j / C::kVStages) & 1u) ^ 1u, p.err, kErrVEmpty, abort_flag)) return;
    mbar_arrive_expect_tx(&sm.v_full[vs], C::kOpBytes);
    for (int c = 0; c < C::kChunks; ++c) {
      uint8_t* dst = sm.v[vs] + c * kChunkBytes;
      tma_load_4d(dst, &maps.v, &sm.v_full[vs], c * 64, t.h, r0, t.b);
      tma_load_4d(dst + kChunkBytes / 2, &maps.v, &sm.v_full[vs], c * 64, t.h, r1, t.b);
    }
  }
}

// Descriptors: one base descriptor per operand buffer; each K step adds a
// compile-time offset to the 14-bit start-address field inside the MMA
// instruction block (addresses stay below 256 KB, so the field never
// carries).  The K steps are expanded with a fold expression.
template <int KK>
constexpr uint32_t kS_off = uint32_t(((KK >> 2) * kChunkBytes + (KK & 3) * 32) >> 4);

template <int... KK>
ICSA_DEV void flat_issue_s_seq(uint64_t q_desc, uint64_t k_desc, uint32_t d_tmem, std::integer_sequence<int, KK...>) {
  constexpr uint32_t idesc = tc::make_idesc_bf16(128, 128, false, false);
  (tc::mma_bf16_ss_off<kS_off<KK>, kS_off<KK>>(d_tmem, q_desc, k_desc, idesc, KK > 0 ? 1u : 0u), ...);
}

template <int D>
ICSA_DEV void flat_issue_s(uint64_t q_desc, uint64_t k_desc, uint32_t d_tmem) {
  flat_issue_s_seq(q_desc, k_desc, d_tmem, std::make_integer_sequence<int, D / 16>{});
}

// P.V: 128 KV rows, 16 per instruction; P occupies 8 TMEM columns per step,
// V advances 16 rows (2048 bytes) per step.
template <int... KK>
ICSA_DEV void flat_issue_pv_seq(uint64_t v_desc, uint32_t p_tmem, uint32_t o_tmem, uint32_t acc,
                                uint32_t idesc, std::integer_sequence<int, KK...>) {
  (tc::mma_bf16_ts_off<uint32_t(KK * 8), uint32_t((KK * 16 * 128) >> 4)>(o_tmem, p_tmem, v_desc, idesc,
                                                                         (KK > 0) ? 1u : acc), ...);
}

template <int D>
ICSA_DEV void flat_issue_pv(uint64_t v_desc, uint32_t p_tmem, uint32_t o_tmem, bool accumulate) {
  flat_issue_pv_seq(v_desc, p_tmem, o_tmem, accumulate ? 1u : 0u, tc::make_idesc_bf16(128, D, false, true),
                    std::make_integer_sequence<int, 8>{});
}

template <int D>
ICSA_DEV void flat_mma(const AttnParams& p, const FTile& t, FSmem<D>& sm, uint32_t tmem) {
  using C = FCfg<D>;
  volatile int* abort_flag = &sm.abort_flag;
  const int n = t.n_steps;
  const uint64_t q0 = tc::make_sw128_desc(smem_u32(sm.q[0]), 16, 1024);
  const uint64_t q1 = tc::make_sw128_desc(smem_u32(sm.q[1]), 16, 1024);
  const uint64_t k0 = tc::make_sw128_desc(smem_u32(sm.k[0]), 16, 1024);
  const uint64_t v0 = tc::make_sw128_desc(smem_u32(sm.v[0]), kChunkBytes, 1024);
  constexpr uint64_t kStageStep = uint64_t(C::kOpBytes >> 4);
  const uint32_t s0 = tmem, s1 = tmem + 256, o0 = tmem + 128, o1 = tmem + 384;
  if (!mbar_wait(&sm.q_full, 0, p.err, kErrQ, abort_flag)) return;
  if (!mbar_wait(&sm.k_full[0], 0, p.err, kErrKFull, abort_flag)) return;
  tc::fence_after_sync();
  flat_issue_s<D>(q0, k0, s0);
  tc::mma_commit(&sm.s_full[0]);
  flat_issue_s<D>(q1, k0, s1);
  tc::mma_commit(&sm.s_full[1]);
  tc::mma_commit(&sm.k_empty[0]);
  int vs = 0, ks = 1 % C::kKStages;
  uint32_t vph = 0, kph = (1 / C::kKStages) & 1;
  for (int j = 0; j < n; ++j) {
    const bool next = j + 1 < n;
    const uint64_t vd = v0 + uint64_t(vs) * kStageStep;
    const uint64_t kd = k0 + uint64_t(ks) * kStageStep;
    if (!mbar_wait(&sm.v_full[vs], vph, p.err, kErrVFull, abort_flag)) return;
    if (!mbar_spin_wait(&sm.p_full[0], uint32_t(j) & 1u, p.err, kErrPFull, abort_flag)) return;
    tc::fence_after_sync();
    flat_issue_pv<D>(vd, s0, o0, j > 0);
    tc::mma_commit(&sm.o_done[0]);
    if (next) {
      if (!mbar_wait(&sm.k_full[ks], kph, p.err, kErrKFull, abort_flag)) return;
      tc::fence_after_sync();
      flat_issue_s<D>(q0, kd, s0);
      tc::mma_commit(&sm.s_full[0]);
    }
    if (!mbar_spin_wait(&sm.p_full[1], uint32_t(j) & 1u, p.err, kErrPFull, abort_flag)) return;
    tc::fence_after_sync();
    flat_issue_pv<D>(vd, s1, o1, j > 0);
    tc::mma_commit(&sm.o_done[1]);
    tc::mma_commit(&sm.v_empty[vs]);
    if (next) {
      flat_issue_s<D>(q1, kd, s1);
      tc::mma_commit(&sm.s_full[1]);
      tc::mma_commit(&sm.k_empty[ks]);
    }
    if (++vs == C::kVStages) { vs = 0; vph ^= 1u; }
    if (++ks == C::kKStages) { ks = 0; kph ^= 1u; }
  }
}

// ---------------------------------------------------------------------------
// Softmax warpgroups (warps 0-3: tile 0, warps 4-7: tile 1) and epilogue.
// ---------------------------------------------------------------------------
template <int D>
ICSA_DEV void flat_softmax(const AttnParams& p, const FTile& t, FSmem<D>& sm, uint32_t tmem) {
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x >> 5;
  const int tile = warp >> 2;
  const int row = threadIdx.x & 127;
  const uint32_t lanes = uint32_t((warp & 3) * 32) << 16;
  const uint32_t s_col = tmem + lanes + tile * 256;
  const uint32_t o_col = s_col + 128;
  const float sl2 = p.scale_log2;
  const int n = t.n_steps;
  float m_ref = -INFINITY, l = 0.f;

  for (int j = 0; j < n; ++j) {
    if (!warp_mbar_wait(&sm.s_full[tile], uint32_t(j) & 1u, p.err, kErrSFull, abort_flag)) return;
    tc::fence_after_sync();
    float s[128];
    tmem_load_row128(s_col, s);
    const int hi = p.tkv - j * 128;  // extended-KV rows beyond tkv are not keys
    if (hi < 128) {
#pragma unroll
      for (int c = 0; c < 128; ++c)
        if (c >= hi) s[c] = -INFINITY;
    }
    const float mx = max128(s);
    const bool need = (mx - m_ref) * sl2 > kRescaleThreshold;
    float alpha = 1.f;
    if (need) {
      alpha = ex2((m_ref - mx) * sl2);
      m_ref = mx;
      l *= alpha;
    }
    const float neg = -m_ref * sl2;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int c = 0; c < 128; c += 4) {
      ffma2(s[c], s[c + 1], s[c], s[c + 1], sl2, sl2, neg, neg);
      ffma2(s[c + 2], s[c + 3], s[c + 2], s[c + 3], sl2, sl2, neg, neg);
      s[c] = ex2(s[c]);
      s[c + 1] = ex2(s[c + 1]);
      s[c + 2] = ex2(s[c + 2]);
      s[c + 3] = ex2(s[c + 3]);
      fadd2(a0, a1, a0, a1, s[c], s[c + 1]);
      fadd2(a2, a3, a2, a3, s[c + 2], s[c + 3]);
      if ((c & 63) == 60) {
        // 64 probabilities done: pack them and write them over S in TMEM
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) pk[e] = pack_bf16x2(s[(c & ~63) + 2 * e], s[(c & ~63) + 2 * e + 1]);
        tc::tmem_st32(s_col + (c >> 6) * 32, pk);
      }
    }
    l += (a0 + a1) + (a2 + a3);
    if (j > 0 && __any_sync(0xffffffffu, need)) {
      // O(j-1) must be complete before it is rescaled
      if (!warp_mbar_wait(&sm.o_done[tile], uint32_t(j - 1) & 1u, p.err, kErrPvDone, abort_flag)) return;
      tc::fence_after_sync();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(o_col + c * 32, r);
        tc::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
        tc::tmem_st32(o_col + c * 32, r);
      }
    }
    tc::tmem_wait_st();
    tc::fence_before_sync();
    mbar_arrive(&sm.p_full[tile]);
  }

  // epilogue
  if (!warp_mbar_wait(&sm.o_done[tile], uint32_t(n - 1) & 1u, p.err, kErrPvDone, abort_flag)) return;
  tc::fence_after_sync();
  const int q = 2 * tile + (row >> 6);
  const int blk = (q == 0) ? t.blk[0] : (q == 1) ? t.blk[1] : (q == 2) ? t.blk[2] : t.blk[3];
  const int wr = (q == 0) ? t.write[0] : (q == 1) ? t.write[1] : (q == 2) ? t.write[2] : t.write[3];
  const int token = blk * kBlock + (row & 63);
  const bool write = wr && token < p.S;
  const float inv = l == 0.f ? 0.f : 1.0f / l;
  const float* oc = p.outc ? p.outc + (size_t(t.bh) * p.NB + blk) * D : nullptr;  // nullptr: no residual term
  const size_t out_row = ((size_t(t.b) * p.S + token) * p.H + t.h) * D;
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    uint32_t r[32];
    __syncwarp();
    tc::tmem_ld32(o_col + c * 32, r);
    tc::tmem_wait_ld();
    float o[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) o[e] = __uint_as_float(r[e]) * inv;
    if (write) store_out32(p, t.b, token, t.h, oc, c * 32, o, out_row);
  }
}

template <int D>
__global__ void __launch_bounds__(kFThreads, 1) flat_kernel(const AttnParams p, const __grid_constant__ AttnMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  FSmem<D>& sm = *reinterpret_cast<FSmem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using C = FCfg<D>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const FTile t = decode_flat_tile(p, blockIdx.x);

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < C::kKStages; ++i) {
      mbar_init(&sm.k_full[i], 1);
      mbar_init(&sm.k_empty[i], 1);
    }
    for (int i = 0; i < C::kVStages; ++i) {
      mbar_init(&sm.v_full[i], 1);
      mbar_init(&sm.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_full[i], 128);
      mbar_init(&sm.o_done[i], 1);
    }
    mbar_init(&sm.mma_fin, 1);
    sm.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kFMmaWarp) {
    tc::tmem_alloc(&sm.tmem_base, kFTmemCols);
    tc::tmem_relinquish();
  }
  if (warp == kFProducerWarp && lane == 0) {
    prefetch_tensormap(&maps.q);
    prefetch_tensormap(&maps.k);
    prefetch_tensormap(&maps.v);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  // Register split: 384 threads launch with 168 registers each; warpgroup 2
  // (producer, MMA issuer, two idle warps) gives registers back so that the
  // softmax warpgroups can hold a whole 128-column row:
  // 256 x 216 + 128 x 72 = 384 x 168.  setmaxnreg is executed by every warp of
  // a warpgroup.
  if (warp < 8) {
    tc::reg_alloc<216>();
    flat_softmax<D>(p, t, sm, tmem);
  } else {
    tc::reg_dealloc<72>();  // one instance for all four warps of warpgroup 2
    if (warp == kFProducerWarp && lane == 0) {
      flat_producer<D>(p, maps, t, sm);
      if (sm.abort_flag) {
        // let copies still in flight land before the shared memory is released
        for (int j = max(0, t.n_steps - C::kKStages); j < t.n_steps; ++j)
          drain_wait(&sm.k_full[j % C::kKStages], uint32_t(j / C::kKStages) & 1u, p.err);
        for (int j = max(0, t.n_steps - C::kVStages); j < t.n_steps; ++j)
          drain_wait(&sm.v_full[j % C::kVStages], uint32_t(j / C::kVStages) & 1u, p.err);
        drain_wait(&sm.q_full, 0, p.err);
      }
    } else if (warp == kFMmaWarp && lane == 0) {
      flat_mma<D>(p, t, sm, tmem);
      tc::mma_commit(&sm.mma_fin);
      drain_wait(&sm.mma_fin, 0, p.err);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kFMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kFTmemCols);
  }
}

}  // namespace

cudaError_t launch_flat_attention(const AttnParams& p, const AttnMaps& maps, int D, cudaStream_t stream) {
  const int ctas = p.B * p.H * ((p.num_flat + 3) / 4);
  if (ctas == 0) return cudaSuccess;
  if (D == 128) return launch_dense_pair_attention(p, maps, stream);
  if (D == 128) {
    const size_t smem = sizeof(FSmem<128>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(flat_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    flat_kernel<128><<<ctas, kFThreads, smem, stream>>>(p, maps);
  } else if (D == 64) {
    const size_t smem = sizeof(FSmem<64>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(flat_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    flat_kernel<64><<<ctas, kFThreads, smem, stream>>>(p, maps);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

ICSA_DEFINE_STICKY_ACCESSOR(sticky_status_flat)

}  // namespace icsa
