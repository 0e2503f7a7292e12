// Stage 3: block attention on the 5th-generation tensor cores.
//
// One kernel serves both halves of the reference's split
// (editing_sparse_attention.py:186-215):
//   * FLAT tiles  -- dense softmax attention of two query blocks (128 rows)
//     over every extended-KV block (the flash_attn_func call, :211-215);
//   * SPARSE tiles -- the fused sparse kernel of the tilelang backend
//     (tilelang_kernels.py:681-997): exact online softmax over the top_k
//     selected extended-KV blocks of each query block, then the "interval"
//     term over all pooled blocks in chunks of 64 (BN = 64) whose
//     contributions g_acc / g_l are, as in the reference, never rescaled.
// and the epilogue writes each row straight to its block's place in the
// [B, S, H, D] output with the residual `+ out_c * alpha` fused in
// (:217-232), so nothing is gathered, scattered or materialised.
//
// Per CTA: one tile of 128 query rows (two 64-token blocks).  Warp roles:
//   warps 0-3  softmax + epilogue; thread t owns row t (= TMEM lane t)
//   warp 4     TMA producer (Q once, then K/V tiles through a ring)
//   warp 5     TMEM allocator and tcgen05.mma issuer
// TMEM columns: S double buffer [0,256), O [256, 256+D), G [384, 384+D).
// Each KV step is 128 rows (two 64-row blocks) of K and V:
//   S = Q K^T     (M=128, N=128, K=D, both operands K-major, SW128)
//   O += P V      (M=128, N=D,   K=128; P K-major in smem, V MN-major)
// In a sparse tile the two query blocks select different KV blocks; step i
// loads block i of each list and a block-diagonal mask keeps rows 0-63 on the
// first 64 columns and rows 64-127 on the last 64, so P V is exact for both.
#include "icsa_kernels.cuh"
#include "icsa_attn_common.cuh"

namespace icsa {

namespace {

using namespace attn;

constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256, kColG = 384;

enum : int { kStepFlat = 0, kStepExact = 1, kStepInterval = 2 };


template <int D>
struct Cfg {
  static constexpr int kStages = (D == 128) ? 2 : 3;
  static constexpr int kOpBytes = 128 * D * 2;  // a 128-row operand tile
  static constexpr int kChunks = D / 64;
};

template <int D>
struct __align__(1024) Smem {
  uint8_t q[Cfg<D>::kOpBytes];
  uint8_t k[Cfg<D>::kStages][Cfg<D>::kOpBytes];
  uint8_t v[Cfg<D>::kStages][Cfg<D>::kOpBytes];
  uint8_t p[2][128 * 128 * 2];
  uint64_t q_full;
  uint64_t k_full[Cfg<D>::kStages], k_empty[Cfg<D>::kStages];
  uint64_t v_full[Cfg<D>::kStages], v_empty[Cfg<D>::kStages];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], pv_done[2];
  uint64_t mma_fin;
  uint32_t tmem_base;
  int abort_flag;
};

// Work description of one CTA.
struct Tile {
  int sparse;       // 0: flat tile, 1: sparse tile
  int bh, b, h;
  int blk[2];       // query blocks (rows 0-63 and 64-127)
  int rank[2];      // rank inside the flat / sparse list
  int write1;       // 0 when the second half duplicates the first (odd count)
  int n_exact;      // exact (or flat) steps
  int n_steps;      // total steps
};

ICSA_DEV Tile decode_tile(const AttnParams& p, int tile) {
  Tile t;
  const int flat_total = p.B * p.H * p.flat_tiles;
  int pair, count, base;
  if (tile < flat_total) {
    t.sparse = 0;
    t.bh = tile / p.flat_tiles;
    pair = tile % p.flat_tiles;
    count = p.num_flat;
    base = 0;
  } else {
    tile -= flat_total;
    t.sparse = 1;
    t.bh = tile / p.sparse_tiles;
    pair = tile % p.sparse_tiles;
    count = p.n_sparse;
    base = p.num_flat;
  }
  t.b = t.bh / p.H;
  t.h = t.bh % p.H;
  t.rank[0] = 2 * pair;
  t.write1 = (2 * pair + 1) < count;
  t.rank[1] = t.write1 ? 2 * pair + 1 : 2 * pair;
  const int* order = p.order + size_t(t.bh) * p.NB + base;
  t.blk[0] = order[t.rank[0]];
  t.blk[1] = order[t.rank[1]];
  if (t.sparse) {
    t.n_exact = p.top_k;
    t.n_steps = p.top_k + p.nkv_pad / 128;
  } else {
    t.n_exact = (p.nkv + 1) / 2;
    t.n_steps = t.n_exact;
  }
  return t;
}

ICSA_DEV int step_kind(const Tile& t, int j) {
  if (!t.sparse) return kStepFlat;
  return j < t.n_exact ? kStepExact : kStepInterval;
}

// First rows (inside the K/V tensors) of the two 64-row halves of KV step j.
ICSA_DEV void step_rows(const AttnParams& p, const Tile& t, int j, int& r0, int& r1) {
  const int* rows = p.kv_rows + size_t(t.bh) * p.nkv;
  if (!t.sparse) {
    r0 = rows[2 * j];
    r1 = (2 * j + 1 < p.nkv) ? rows[2 * j + 1] : r0;  // missing half: any valid rows, masked
  } else {
    const int* idx = p.sparse_idx + size_t(t.bh) * p.n_sparse * p.top_k;
    r0 = rows[idx[size_t(t.rank[0]) * p.top_k + j]];
    r1 = rows[idx[size_t(t.rank[1]) * p.top_k + j]];
  }
}

// ---------------------------------------------------------------------------
// Warp 4, one thread: TMA producer.
// ---------------------------------------------------------------------------
template <int D>
ICSA_DEV void run_producer(const AttnParams& p, const AttnMaps& maps, const Tile& t, Smem<D>& sm) {
  using C = Cfg<D>;
  volatile int* abort_flag = &sm.abort_flag;
  // Q: two 64-row blocks per 64-wide D chunk (8 KB each).
  mbar_arrive_expect_tx(&sm.q_full, C::kOpBytes);
  for (int c = 0; c < C::kChunks; ++c)
    for (int half = 0; half < 2; ++half)
      tma_load_4d(sm.q + c * kChunkBytes + half * (kChunkBytes / 2), &maps.q, &sm.q_full, c * 64, t.h,
                  t.blk[half] * kBlock, t.b);

  for (int j = 0; j < t.n_steps; ++j) {
    const int st = j % C::kStages;
    const uint32_t ph = uint32_t(j / C::kStages) & 1u;
    const int kind = step_kind(t, j);
    int r0 = 0, r1 = 0, ichunk = 0;
    if (kind == kStepInterval)
      ichunk = j - t.n_exact;  // 128 pooled rows per step
    else
      step_rows(p, t, j, r0, r1);

    if (!mbar_wait(&sm.k_empty[st], ph ^ 1u, p.err, kErrKEmpty, abort_flag)) break;
    mbar_arrive_expect_tx(&sm.k_full[st], C::kOpBytes);
    for (int c = 0; c < C::kChunks; ++c) {
      uint8_t* dst = sm.k[st] + c * kChunkBytes;
      if (kind == kStepInterval) {
        tma_load_3d(dst, &maps.kc, &sm.k_full[st], c * 64, ichunk * 128, t.bh);
      } else {
        tma_load_4d(dst, &maps.k, &sm.k_full[st], c * 64, t.h, r0, t.b);
        tma_load_4d(dst + kChunkBytes / 2, &maps.k, &sm.k_full[st], c * 64, t.h, r1, t.b);
      }
    }
    if (!mbar_wait(&sm.v_empty[st], ph ^ 1u, p.err, kErrVEmpty, abort_flag)) break;
    mbar_arrive_expect_tx(&sm.v_full[st], C::kOpBytes);
    for (int c = 0; c < C::kChunks; ++c) {
      uint8_t* dst = sm.v[st] + c * kChunkBytes;
      if (kind == kStepInterval) {
        tma_load_3d(dst, &maps.vc, &sm.v_full[st], c * 64, ichunk * 128, t.bh);
      } else {
        tma_load_4d(dst, &maps.v, &sm.v_full[st], c * 64, t.h, r0, t.b);
        tma_load_4d(dst + kChunkBytes / 2, &maps.v, &sm.v_full[st], c * 64, t.h, r1, t.b);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Warp 5, one thread: tcgen05.mma issuer.
// ---------------------------------------------------------------------------
template <int D>
ICSA_DEV void issue_pv(const AttnParams& p, const Tile& t, Smem<D>& sm, uint32_t tmem, int i) {
  using C = Cfg<D>;
  volatile int* abort_flag = &sm.abort_flag;
  const int st = i % C::kStages;
  const int pb = i & 1;
  if (!mbar_wait(&sm.v_full[st], uint32_t(i / C::kStages) & 1u, p.err, kErrVFull, abort_flag)) return;
  if (!mbar_wait(&sm.p_full[pb], uint32_t(i >> 1) & 1u, p.err, kErrPFull, abort_flag)) return;
  tc::fence_after_sync();
  const bool interval = step_kind(t, i) == kStepInterval;
  const uint32_t acc_col = interval ? kColG : kColO;
  const int first = interval ? t.n_exact : 0;
  constexpr uint32_t idesc = tc::make_idesc_bf16(128, D, false, true);
  const uint32_t p_addr = smem_u32(sm.p[pb]);
  const uint32_t v_addr = smem_u32(sm.v[st]);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {  // K = 128 KV rows, 16 per instruction
    const uint64_t a = tc::make_sw128_desc(p_addr + (kk >> 2) * kChunkBytes + (kk & 3) * 32, 16, 1024);
    const uint64_t b = tc::make_sw128_desc(v_addr + kk * 16 * 128, kChunkBytes, 1024);
    tc::mma_bf16_ss(tmem + acc_col, a, b, idesc, (i > first || kk > 0) ? 1u : 0u);
  }
  tc::mma_commit(&sm.pv_done[pb]);
  tc::mma_commit(&sm.v_empty[st]);
}

template <int D>
ICSA_DEV void run_mma(const AttnParams& p, const Tile& t, Smem<D>& sm, uint32_t tmem) {
  using C = Cfg<D>;
  volatile int* abort_flag = &sm.abort_flag;
  if (!mbar_wait(&sm.q_full, 0, p.err, kErrQ, abort_flag)) return;
  constexpr uint32_t idesc = tc::make_idesc_bf16(128, 128, false, false);
  const uint32_t q_addr = smem_u32(sm.q);
  for (int j = 0; j < t.n_steps; ++j) {
    const int st = j % C::kStages;
    const int sb = j & 1;
    if (!mbar_wait(&sm.k_full[st], uint32_t(j / C::kStages) & 1u, p.err, kErrKFull, abort_flag)) return;
    if (j >= 2 && !mbar_wait(&sm.s_empty[sb], uint32_t((j >> 1) - 1) & 1u, p.err, kErrSEmpty, abort_flag)) return;
    tc::fence_after_sync();
    const uint32_t k_addr = smem_u32(sm.k[st]);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t off = (kk >> 2) * kChunkBytes + (kk & 3) * 32;
      const uint64_t a = tc::make_sw128_desc(q_addr + off, 16, 1024);
      const uint64_t b = tc::make_sw128_desc(k_addr + off, 16, 1024);
      tc::mma_bf16_ss(tmem + kColS + sb * 128, a, b, idesc, kk > 0 ? 1u : 0u);
    }
    tc::mma_commit(&sm.s_full[sb]);
    tc::mma_commit(&sm.k_empty[st]);
    if (j >= 1) issue_pv<D>(p, t, sm, tmem, j - 1);
    if (*abort_flag) return;
  }
  if (t.n_steps > 0) issue_pv<D>(p, t, sm, tmem, t.n_steps - 1);
}

// ---------------------------------------------------------------------------
// Warps 0-3: softmax.  Thread t owns query row t of the tile.
// ---------------------------------------------------------------------------
// Store one row of P (128 bf16) into the SW128 K-major P tile: two 64-wide
// chunks of [128 rows][128 B]; 16-byte piece i of row r sits at slot i ^ (r & 7).
ICSA_DEV void store_p_row(uint8_t* ptile, int row, const float (&pr)[128]) {
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    uint8_t* base = ptile + ch * kChunkBytes + row * 128;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float* v = pr + ch * 64 + i * 8;
      uint4 u;
      u.x = pack_bf16x2(v[0], v[1]);
      u.y = pack_bf16x2(v[2], v[3]);
      u.z = pack_bf16x2(v[4], v[5]);
      u.w = pack_bf16x2(v[6], v[7]);
      *reinterpret_cast<uint4*>(base + ((i ^ (row & 7)) << 4)) = u;
    }
  }
}

struct RowState {
  float m_ref;   // max used as the exponent origin of O and l (raw score units)
  float m_true;  // true running max (raw units), as the reference tracks it
  float l;       // softmax denominator of the exact / flat part, relative to m_ref
  float g_l;     // interval denominator (never rescaled)
};

template <int D>
ICSA_DEV void run_softmax(const AttnParams& p, const Tile& t, Smem<D>& sm, uint32_t tmem, RowState& rs) {
  volatile int* abort_flag = &sm.abort_flag;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int half = tid >> 6;  // query block of this row
  const uint32_t lane_base = uint32_t(warp * 32) << 16;
  const float sl2 = p.scale_log2;
  const int words = p.nkv_pad / 32;
  const uint32_t* mask_row =
      t.sparse ? p.sel_mask + (size_t(t.bh) * p.n_sparse + (half ? t.rank[1] : t.rank[0])) * words : nullptr;
  rs.m_ref = -INFINITY;
  rs.m_true = -INFINITY;
  rs.l = 0.f;
  rs.g_l = 0.f;

  for (int j = 0; j < t.n_steps; ++j) {
    const int sb = j & 1;
    if (!warp_mbar_wait(&sm.s_full[sb], uint32_t(j >> 1) & 1u, p.err, kErrSFull, abort_flag)) return;
    tc::fence_after_sync();
    float s[128];
    tmem_load_row128(tmem + lane_base + kColS + sb * 128, s);
    tc::fence_before_sync();
    mbar_arrive(&sm.s_empty[sb]);

    const int kind = step_kind(t, j);
    float alpha = 1.f;
    bool need = false;
    if (kind != kStepInterval) {
      // valid columns [lo, hi)
      int lo = 0, hi = 128;
      if (kind == kStepExact) {
        lo = half * 64;
        hi = lo + 64;
      } else {
        hi = min(128, p.tkv - j * 128);
      }
#pragma unroll
      for (int c = 0; c < 128; ++c)
        if (c < lo || c >= hi) s[c] = -INFINITY;
      const float mx = max128(s);
      rs.m_true = fmaxf(rs.m_true, mx);
      need = (mx - rs.m_ref) * sl2 > kRescaleThreshold;
      if (need) {
        alpha = exp2f((rs.m_ref - rs.m_true) * sl2);
        rs.m_ref = rs.m_true;
        rs.l *= alpha;
      }
      const float neg = -rs.m_ref * sl2;
      float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const float e = ex2(fmaf(s[c], sl2, neg));  // masked: 2^-inf = 0
        s[c] = e;
        part[c & 7] += e;
      }
      rs.l += ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
    } else {
      // Interval term: two BN=64 chunks of pooled blocks per step.
      const int ci = j - t.n_exact;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int chunk = 2 * ci + hh;
        const uint32_t w0 = mask_row[chunk * 2], w1 = mask_row[chunk * 2 + 1];
        float cm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int blk = chunk * 64 + c;
          const uint32_t w = c < 32 ? w0 : w1;
          const bool valid = blk < p.nkv && !((w >> (c & 31)) & 1u);
          const float x = s[hh * 64 + c] * (1.0f / 64.0f);
          s[hh * 64 + c] = valid ? x : -INFINITY;
          cm[c & 3] = fmaxf(cm[c & 3], s[hh * 64 + c]);
        }
        rs.m_true = fmaxf(rs.m_true, fmaxf(fmaxf(cm[0], cm[1]), fmaxf(cm[2], cm[3])));
        const float neg = -rs.m_true * sl2;
        float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float x = s[hh * 64 + c];
          const float e = (x == -INFINITY) ? 0.f : ex2(fmaf(x, sl2, neg));
          s[hh * 64 + c] = e;
          part[c & 3] += e;
        }
        rs.g_l += ((part[0] + part[1]) + (part[2] + part[3])) * 64.0f;
      }
    }

    const int pb = j & 1;
    if (j >= 2 && !warp_mbar_wait(&sm.pv_done[pb], uint32_t((j - 2) >> 1) & 1u, p.err, kErrPvDone, abort_flag)) return;
    if (kind != kStepInterval && j > 0 && __any_sync(0xffffffffu, need)) {
      if (!warp_mbar_wait(&sm.pv_done[(j - 1) & 1], uint32_t((j - 1) >> 1) & 1u, p.err, kErrPvDone, abort_flag)) return;
      tc::fence_after_sync();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        const uint32_t taddr = tmem + lane_base + kColO + c * 32;
        tc::tmem_ld32(taddr, r);
        tc::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
        tc::tmem_st32(taddr, r);
      }
      tc::tmem_wait_st();
    }
    store_p_row(sm.p[pb], tid, s);
    fence_proxy_async_smem();
    tc::fence_before_sync();
    mbar_arrive(&sm.p_full[pb]);
  }
}

// ---------------------------------------------------------------------------
// Epilogue: normalise, round to bf16 as the reference's attention outputs
// are, add the compressed-attention residual and store the row in place.
// ---------------------------------------------------------------------------
template <int D>
ICSA_DEV void run_epilogue(const AttnParams& p, const Tile& t, Smem<D>& sm, uint32_t tmem, const RowState& rs) {
  volatile int* abort_flag = &sm.abort_flag;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int half = tid >> 6;
  const uint32_t lane_base = uint32_t(warp * 32) << 16;
  const int last = t.n_steps - 1;
  if (!warp_mbar_wait(&sm.pv_done[last & 1], uint32_t(last >> 1) & 1u, p.err, kErrPvDone, abort_flag)) return;
  tc::fence_after_sync();

  const int blk = half ? t.blk[1] : t.blk[0];
  const int token = blk * kBlock + (tid & 63);
  const bool write = (half == 0 || t.write1) && token < p.S;
  float f = 1.f, denom = rs.l;
  if (t.sparse) {
    f = exp2f((rs.m_ref - rs.m_true) * p.scale_log2);
    denom = rs.l * f + rs.g_l;
  }
  const float* oc = p.outc + (size_t(t.bh) * p.NB + blk) * D;
  const size_t out_row = ((size_t(t.b) * p.S + token) * p.H + t.h) * D;
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    uint32_t ro[32], rg[32];
    __syncwarp();
    tc::tmem_ld32(tmem + lane_base + kColO + c * 32, ro);
    if (t.sparse) tc::tmem_ld32(tmem + lane_base + kColG + c * 32, rg);
    tc::tmem_wait_ld();
    float o[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      float acc = __uint_as_float(ro[e]);
      if (t.sparse) acc = acc * f + __uint_as_float(rg[e]);
      o[e] = denom == 0.f ? 0.f : __fdiv_rn(acc, denom);
    }
    if (write) store_out32(p, t.b, token, t.h, oc, c * 32, o, out_row);
  }
}

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads, 1) attn_kernel(const AttnParams p, const __grid_constant__ AttnMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using C = Cfg<D>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Tile t = decode_tile(p, blockIdx.x);

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&sm.k_full[i], 1);
      mbar_init(&sm.v_full[i], 1);
      mbar_init(&sm.k_empty[i], 1);
      mbar_init(&sm.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_empty[i], kSoftmaxThreads);
      mbar_init(&sm.p_full[i], kSoftmaxThreads);
      mbar_init(&sm.pv_done[i], 1);
    }
    mbar_init(&sm.mma_fin, 1);
    sm.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tensormap(&maps.q);
    prefetch_tensormap(&maps.k);
    prefetch_tensormap(&maps.v);
    if (t.sparse) {
      prefetch_tensormap(&maps.kc);
      prefetch_tensormap(&maps.vc);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  if (warp < 4) {
    RowState rs;
    run_softmax<D>(p, t, sm, tmem, rs);
    run_epilogue<D>(p, t, sm, tmem, rs);
  } else if (warp == kProducerWarp) {
    if (lane == 0) {
      run_producer<D>(p, maps, t, sm);
      // Let every copy this CTA issued land before its shared memory goes.
      const int issued = t.n_steps;
      for (int j = max(0, issued - C::kStages); j < issued; ++j) {
        const int st = j % C::kStages;
        const uint32_t ph = uint32_t(j / C::kStages) & 1u;
        if (sm.abort_flag) {
          drain_wait(&sm.k_full[st], ph, p.err);
          drain_wait(&sm.v_full[st], ph, p.err);
        }
      }
      if (sm.abort_flag) drain_wait(&sm.q_full, 0, p.err);
    }
  } else {
    if (lane == 0) {
      run_mma<D>(p, t, sm, tmem);
      // All MMAs of this CTA complete before TMEM is released.
      tc::mma_commit(&sm.mma_fin);
      drain_wait(&sm.mma_fin, 0, p.err);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_attention(const AttnParams& p, const AttnMaps& maps, int D, cudaStream_t stream) {
  const int tiles = p.B * p.H * (p.flat_tiles + p.sparse_tiles);
  if (tiles == 0) return cudaSuccess;
  if (D == 128) {
    const size_t smem = sizeof(Smem<128>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    attn_kernel<128><<<tiles, kThreads, smem, stream>>>(p, maps);
  } else if (D == 64) {
    const size_t smem = sizeof(Smem<64>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    attn_kernel<64><<<tiles, kThreads, smem, stream>>>(p, maps);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace icsa
