// Block-sparse attention for the "sparse" query blocks: the reference's
// fused tilelang kernel (tilelang_kernels.py:681-997, driven by
// tilelang_host.py:121-206), fused with the scatter and residual of
// editing_sparse_attention.py:217-232.
//
// Per query block the reference computes
//   (a) exact online softmax over its top_k selected 64-row KV blocks;
//   (b) an "interval" term over all pooled KV blocks in chunks of BN = 64:
//       logits q.KC/64 (KC = block sums), selected blocks and blocks >= nkv
//       masked, running max updated per chunk (rescaling acc/l of (a)), and
//       probabilities weighted x64 accumulated into g_l / g_acc WITHOUT
//       rescaling when a later chunk raises the max;
//   (c) out = (acc + g_acc) / (l + g_l), 0 where the denominator is 0.
//
// Per CTA: one 128-row tile = two sparse query blocks A (rows 0-63) and B
// (rows 64-127).  Exact step i loads block i of A's list into KV rows 0-63
// and block i of B's list into rows 64-127; the score tile is then
// block-diagonal (rows of A only use columns 0-63, rows of B columns 64-127)
// and P is written with zeros off the diagonal, so one M=128 x N=128 x K=128
// P.V computes both.  Interval steps load 128 pooled rows (two BN=64 chunks).
//
// Roles: warps 0-3 softmax + epilogue (thread t <-> row t <-> TMEM lane t);
// warp 4 TMA producer; warp 5 TMEM allocator + MMA issuer.
// TMEM: S double buffer [0,128) [128,256), O [256,256+D) for the exact part,
// G [384,384+D) for the interval part.  P of exact step j goes to buffer j%2
// at [384 + 64 (j%2), +64): G's columns are idle until the interval steps,
// and there each row's other-block half of P stays zero from one store at
// the start instead of being rewritten every step.  P of an interval step
// overwrites the first 64 columns of its S buffer.  The MMA thread issues
// S(j+1) before P(j).V so the tensor core computes the next scores while the
// softmax of step j runs; S(j) complete implies P.V(j-2) complete, so P(j)
// never overwrites a buffer still being read.
#include "icsa_attn_common.cuh"

#include <utility>

namespace icsa {

namespace {

using namespace attn;

constexpr int kSThreads = 192;
constexpr int kSProducerWarp = 4;
constexpr int kSMmaWarp = 5;
constexpr uint32_t kSTmemCols = 512;
constexpr uint32_t kSColO = 256, kSColG = 384;
constexpr int kSMaskWords = 64;  // masks of up to 2048 extended-KV blocks are staged in shared memory

template <int D>
struct SCfg {
  static constexpr int kOpBytes = 128 * D * 2;
  static constexpr int kChunks = D / 64;
  static constexpr int kStages = (D == 128) ? 3 : 6;
};

template <int D>
struct __align__(1024) SSmem {
  uint8_t q[SCfg<D>::kOpBytes];
  uint8_t k[SCfg<D>::kStages][SCfg<D>::kOpBytes];
  uint8_t v[SCfg<D>::kStages][SCfg<D>::kOpBytes];
  uint64_t q_full;
  uint64_t k_full[SCfg<D>::kStages];
  uint64_t v_full[SCfg<D>::kStages], v_empty[SCfg<D>::kStages];
  float outc[2][D];                       // out_compress rows of the tile's two query blocks
  uint32_t mask[2][kSMaskWords];          // their selection bit masks (when nkv_pad <= 32 * kSMaskWords)
  uint64_t s_full[2], p_full[2];          // p_full per S buffer: the softmax may run one step ahead
  uint64_t mma_fin;
  uint32_t tmem_base;
  int abort_flag;
};

static_assert(sizeof(SSmem<128>) + 1024 <= 232448, "sparse kernel shared memory exceeds 227 KB");
static_assert(sizeof(SSmem<64>) + 1024 <= 232448, "sparse kernel shared memory exceeds 227 KB");

struct STile {
  int bh, b, h;
  int blk[2];   // query blocks of rows [0,64) and [64,128)
  int rank[2];  // their ranks in the sparse list
  int write1;   // 0 when block B duplicates A (odd count)
  int n_exact, n_steps;
};

ICSA_DEV STile decode_sparse_tile(const AttnParams& p, int cta) {
  STile t;
  t.bh = cta / p.sparse_tiles;
  const int pair = cta % p.sparse_tiles;
  t.b = t.bh / p.H;
  t.h = t.bh % p.H;
  t.rank[0] = 2 * pair;
  t.write1 = 2 * pair + 1 < p.n_sparse;
  t.rank[1] = t.write1 ? 2 * pair + 1 : 2 * pair;
  const int* order = p.order + size_t(t.bh) * p.NB + p.num_flat;
  t.blk[0] = order[t.rank[0]];
  t.blk[1] = order[t.rank[1]];
  t.n_exact = p.top_k;
  t.n_steps = p.top_k + p.nkv_pad / 128;
  return t;
}

template <int D>
ICSA_DEV void sparse_producer(const AttnParams& p, const AttnMaps& maps, const STile& t, SSmem<D>& sm) {
  using C = SCfg<D>;
  volatile int* abort_flag = &sm.abort_flag;
  mbar_arrive_expect_tx(&sm.q_full, C::kOpBytes);
  for (int c = 0; c < C::kChunks; ++c)
    for (int half = 0; half < 2; ++half)
      tma_load_4d(sm.q + c * kChunkBytes + half * (kChunkBytes / 2), &maps.q, &sm.q_full, c * 64, t.h,
                  t.blk[half] * kBlock, t.b);
  const int* rows = p.kv_rows + size_t(t.bh) * p.nkv;
  const int* idx = p.sparse_idx + size_t(t.bh) * p.n_sparse * p.top_k;
  const int* idx0 = idx + size_t(t.rank[0]) * p.top_k;
  const int* idx1 = idx + size_t(t.rank[1]) * p.top_k;
  for (int j = 0; j < t.n_steps; ++j) {
    const int st = j % C::kStages;
    const uint32_t ph = (uint32_t(j / C::kStages) & 1u) ^ 1u;
    const bool exact = j < t.n_exact;
    int r0 = 0, r1 = 0;
    if (exact) {
      r0 = rows[idx0[j]];
      r1 = rows[idx1[j]];
    }
    const int prow = (j - t.n_exact) * 128;  // interval: pooled rows
    // a stage is free once the P.V that read its values is done (its S,
    // issued earlier, is done then too): one barrier frees both halves
    if (!mbar_wait(&sm.v_empty[st], ph, p.err, kErrVEmpty, abort_flag)) return;
    mbar_arrive_expect_tx(&sm.k_full[st], C::kOpBytes);
    for (int c = 0; c < C::kChunks; ++c) {
      uint8_t* dst = sm.k[st] + c * kChunkBytes;
      if (exact) {
        tma_load_4d(dst, &maps.k, &sm.k_full[st], c * 64, t.h, r0, t.b);
        tma_load_4d(dst + kChunkBytes / 2, &maps.k, &sm.k_full[st], c * 64, t.h, r1, t.b);
      } else {
        tma_load_3d(dst, &maps.kc, &sm.k_full[st], c * 64, prow, t.bh);
      }
    }
    mbar_arrive_expect_tx(&sm.v_full[st], C::kOpBytes);
    for (int c = 0; c < C::kChunks; ++c) {
      uint8_t* dst = sm.v[st] + c * kChunkBytes;
      if (exact) {
        tma_load_4d(dst, &maps.v, &sm.v_full[st], c * 64, t.h, r0, t.b);
        tma_load_4d(dst + kChunkBytes / 2, &maps.v, &sm.v_full[st], c * 64, t.h, r1, t.b);
      } else {
        tma_load_3d(dst, &maps.vc, &sm.v_full[st], c * 64, prow, t.bh);
      }
    }
  }
}

// Descriptor offsets of the K steps (16 bf16 = 32 bytes inside a 128-byte
// swizzled row; the next 64-wide chunk of d is 16 KB further), added inside
// the instruction block so that no per-step descriptor is built.
template <int KK>
constexpr uint32_t kSparseSOff = uint32_t(((KK >> 2) * kChunkBytes + (KK & 3) * 32) >> 4);

template <int... KK>
ICSA_DEV void sparse_issue_s_seq(uint64_t q_desc, uint64_t k_desc, uint32_t d_tmem, std::integer_sequence<int, KK...>) {
  constexpr uint32_t idesc = tc::make_idesc_bf16(128, 128, false, false);
  (tc::mma_bf16_ss_elect<kSparseSOff<KK>, kSparseSOff<KK>>(d_tmem, q_desc, k_desc, idesc, KK > 0 ? 1u : 0u), ...);
}

// P.V: 128 KV rows, 16 per instruction; P occupies 8 TMEM columns per step,
// V (MN-major) advances 16 rows = 2048 bytes.
template <int D, int... KK>
ICSA_DEV void sparse_issue_pv_seq(uint64_t v_desc, uint32_t p_tmem, uint32_t o_tmem, uint32_t acc,
                                  std::integer_sequence<int, KK...>) {
  constexpr uint32_t idesc = tc::make_idesc_bf16(128, D, false, true);
  (tc::mma_bf16_ts_elect<uint32_t(KK * 8), uint32_t((KK * 16 * 128) >> 4)>(o_tmem, p_tmem, v_desc, idesc,
                                                                           (KK > 0) ? 1u : acc),
   ...);
}

// MMA issuer: all 32 lanes of warp 5 run this loop (waits are warp-uniform,
// one elected lane issues each instruction).
template <int D>
ICSA_DEV void sparse_mma(const AttnParams& p, const STile& t, SSmem<D>& sm, uint32_t tmem) {
  using C = SCfg<D>;
  volatile int* abort_flag = &sm.abort_flag;
  const int n = t.n_steps;
  const uint64_t qd = tc::make_sw128_desc(smem_u32(sm.q), 16, 1024);
  const uint64_t kd0 = tc::make_sw128_desc(smem_u32(sm.k[0]), 16, 1024);
  const uint64_t vd0 = tc::make_sw128_desc(smem_u32(sm.v[0]), kChunkBytes, 1024);
  constexpr uint64_t kStageStep = uint64_t(C::kOpBytes >> 4);
  if (!warp_mbar_wait(&sm.q_full, 0, p.err, kErrQ, abort_flag)) return;
  auto issue_s = [&](int j) -> bool {
    const int st = j % C::kStages;
    if (!warp_mbar_wait(&sm.k_full[st], uint32_t(j / C::kStages) & 1u, p.err, kErrKFull, abort_flag)) return false;
    tc::fence_after_sync();
    sparse_issue_s_seq(qd, kd0 + uint64_t(st) * kStageStep, tmem + uint32_t(j & 1) * 128u,
                       std::make_integer_sequence<int, D / 16>{});
    tc::mma_commit_elect(&sm.s_full[j & 1]);
    return true;
  };
  if (!issue_s(0)) return;
  for (int j = 0; j < n; ++j) {
    // S(j+1) goes to the buffer of P(j-1), whose P.V was issued before
    if (j + 1 < n && !issue_s(j + 1)) return;
    const int st = j % C::kStages;
    if (!warp_mbar_wait(&sm.v_full[st], uint32_t(j / C::kStages) & 1u, p.err, kErrVFull, abort_flag)) return;
    if (!warp_mbar_wait(&sm.p_full[j & 1], uint32_t(j >> 1) & 1u, p.err, kErrPFull, abort_flag)) return;
    tc::fence_after_sync();
    const bool interval = j >= t.n_exact;
    const uint32_t acc = interval ? (j > t.n_exact) : (j > 0);
    sparse_issue_pv_seq<D>(vd0 + uint64_t(st) * kStageStep,
                           interval ? tmem + uint32_t(j & 1) * 128u : tmem + kSColG + uint32_t(j & 1) * 64u,
                           tmem + (interval ? kSColG : kSColO), acc ? 1u : 0u, std::make_integer_sequence<int, 8>{});
    // v_empty also tells the softmax that P.V(j) is done (before an O rescale)
    tc::mma_commit_elect(&sm.v_empty[st]);
  }
}

// ---------------------------------------------------------------------------
// Softmax (warps 0-3) and epilogue.  Warps 0-1 hold the rows of block A,
// warps 2-3 those of block B, so the block-diagonal half a row needs is
// warp-uniform.
// ---------------------------------------------------------------------------
ICSA_DEV float max64(const float (&s)[64]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(s[i], s[i + 8]);
#pragma unroll
  for (int c = 16; c < 64; c += 16)
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmax3(m[i], s[c + i], s[c + 8 + i]);
  return fmax3(fmax3(m[0], m[1], m[2]), fmax3(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// The four softmax warps meet at named barrier 1 (staged masks and
// out_compress), so none may leave early: after a failed wait the abort flag
// is set, later waits return at once, the loop runs on over stale data and
// the error code marks the result invalid.
template <int D>
ICSA_DEV void sparse_softmax(const AttnParams& p, const AttnMaps& maps, const STile& t, SSmem<D>& sm, uint32_t tmem) {
  volatile int* abort_flag = &sm.abort_flag;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int half = warp >> 1;
  const uint32_t lanes = uint32_t(warp * 32) << 16;
  const float sl2 = p.scale_log2;
  const int n = t.n_steps;
  const int words = p.nkv_pad / 32;
  // Stage what the interval steps and the epilogue read (masks, out_compress)
  // in shared memory; the loads are issued now and land while the exact
  // steps run.  The four softmax warps meet at named barrier 1 before use.
  const bool mask_in_smem = words <= kSMaskWords;
  {
    const int hb = tid >> 6, i = tid & 63;
    const int rk = hb ? t.rank[1] : t.rank[0];
    const int bk = hb ? t.blk[1] : t.blk[0];
    const float* oc_src = p.outc + (size_t(t.bh) * p.NB + bk) * D;
    // scalar alpha: the residual term out_c * alpha of the block, rounded as the
    // reference rounds it; tensor alpha: out_c itself (alpha varies by token)
    const bool scalar = p.alpha_mode == ICSA_ALPHA_SCALAR;
    for (int d = i; d < D; d += 64) sm.outc[hb][d] = scalar ? ca_scalar(p, oc_src[d]) : oc_src[d];
    if (mask_in_smem) {
      const uint32_t* msrc = p.sel_mask + (size_t(t.bh) * p.n_sparse + rk) * words;
      for (int w = i; w < words; w += 64) sm.mask[hb][w] = msrc[w];
    }
  }
  const uint32_t* mask_row = mask_in_smem ? sm.mask[half]
                                          : p.sel_mask + (size_t(t.bh) * p.n_sparse + (half ? t.rank[1] : t.rank[0])) * words;
  {
    // exact-step P buffers b = 0, 1 live in G's columns [64 b, 64 b + 64)
    // until the interval steps; the other block's half of each stays zero
    uint32_t zero[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) zero[e] = 0u;
    tc::tmem_st32(tmem + lanes + kSColG + (1 - half) * 32, zero);
    tc::tmem_st32(tmem + lanes + kSColG + 64u + (1 - half) * 32, zero);
  }
  bool staged = false;
  float m_ref = -INFINITY;   // exponent origin of O and l (raw score units)
  float m_true = -INFINITY;  // running max as the reference tracks it
  float l = 0.f, g_l = 0.f;

  for (int j = 0; j < n; ++j) {
    const int sb = j & 1;
    warp_mbar_wait(&sm.s_full[sb], uint32_t(j >> 1) & 1u, p.err, kErrSFull, abort_flag);
    tc::fence_after_sync();
    const uint32_t s_col = tmem + lanes + sb * 128;
    if (j < t.n_exact) {
      // exact step: this row's 64 keys are columns [64*half, 64*half+64)
      float s[64];
      {
        uint32_t r[2][32];
        tc::tmem_ld32(s_col + half * 64, r[0]);
        tc::tmem_ld32(s_col + half * 64 + 32, r[1]);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 64; ++c) s[c] = __uint_as_float(r[c >> 5][c & 31]);
      }
      const float mx = max64(s);
      m_true = fmaxf(m_true, mx);
      const bool need = (mx - m_ref) * sl2 > kRescaleThreshold;
      float alpha = 1.f;
      if (need) {
        alpha = ex2((m_ref - m_true) * sl2);
        m_ref = m_true;
        l *= alpha;
      }
      const float neg = -m_ref * sl2;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 4) {
        ffma2(s[c], s[c + 1], s[c], s[c + 1], sl2, sl2, neg, neg);
        ffma2(s[c + 2], s[c + 3], s[c + 2], s[c + 3], sl2, sl2, neg, neg);
        s[c] = ex2(s[c]);
        s[c + 1] = ex2(s[c + 1]);
        s[c + 2] = ex2(s[c + 2]);
        s[c + 3] = ex2(s[c + 3]);
        fadd2(a0, a1, a0, a1, s[c], s[c + 1]);
        fadd2(a2, a3, a2, a3, s[c + 2], s[c + 3]);
      }
      l += (a0 + a1) + (a2 + a3);
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // P.V(j-1) done: the completion of v_empty for its stage.  S(j) is
        // complete, so P.V(j-2) is too (the tensor core runs in issue order)
        // and P.V(j+2), the stage's next user, cannot have run: the parity
        // names exactly P.V(j-1).
        warp_mbar_wait(&sm.v_empty[(j - 1) % SCfg<D>::kStages], uint32_t((j - 1) / SCfg<D>::kStages) & 1u, p.err,
                       kErrPvDone, abort_flag);
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tc::tmem_ld32(tmem + lanes + kSColO + c * 32, r);
          tc::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
          tc::tmem_st32(tmem + lanes + kSColO + c * 32, r);
        }
      }
      uint32_t pk[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) pk[e] = pack_bf16x2(s[2 * e], s[2 * e + 1]);
      tc::tmem_st32(tmem + lanes + kSColG + uint32_t(sb) * 64u + half * 32, pk);
    } else {
      if (!staged) {
        asm volatile("bar.sync 1, 128;" ::: "memory");
        staged = true;
      }
      // interval step: two BN=64 chunks of pooled blocks, all 128 columns.
      // Logits are q.KC / 64; dividing by 64 is exact, so the maxima are
      // taken on the raw scores and 1/64 is folded into the exponent's
      // multiplier.  Both chunks are masked and reduced first, then both
      // exponentiated (chunk 1 uses the maximum after chunk 0, as the
      // reference updates it chunk by chunk).
      float s[128];
      tmem_load_row128(s_col, s);
      const int ci = j - t.n_exact;
      float cmax[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int chunk = 2 * ci + hh;
        const int lim = p.nkv - chunk * 64;  // columns >= lim are beyond the extended KV
        const uint32_t w0 = mask_row[2 * chunk], w1 = mask_row[2 * chunk + 1];
        float cm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const uint32_t w = c < 32 ? w0 : w1;
          const bool valid = c < lim && !((w >> (c & 31)) & 1u);
          const float x = valid ? s[hh * 64 + c] : -INFINITY;
          s[hh * 64 + c] = x;
          cm[c & 3] = fmaxf(cm[c & 3], x);
        }
        cmax[hh] = fmaxf(fmaxf(cm[0], cm[1]), fmaxf(cm[2], cm[3])) * (1.0f / 64.0f);
      }
      const float m0 = fmaxf(m_true, cmax[0]);
      const float m1 = fmaxf(m0, cmax[1]);
      m_true = m1;
      const float sl2b = sl2 * (1.0f / 64.0f);
      const float neg[2] = {-m0 * sl2, -m1 * sl2};
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int c = 0; c < 64; c += 4) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float* x = s + hh * 64 + c;
          ffma2(x[0], x[1], x[0], x[1], sl2b, sl2b, neg[hh], neg[hh]);
          ffma2(x[2], x[3], x[2], x[3], sl2b, sl2b, neg[hh], neg[hh]);
          x[0] = ex2(x[0]);
          x[1] = ex2(x[1]);
          x[2] = ex2(x[2]);
          x[3] = ex2(x[3]);
          fadd2(acc[hh][0], acc[hh][1], acc[hh][0], acc[hh][1], x[0], x[1]);
          fadd2(acc[hh][2], acc[hh][3], acc[hh][2], acc[hh][3], x[2], x[3]);
        }
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) g_l += ((acc[hh][0] + acc[hh][1]) + (acc[hh][2] + acc[hh][3])) * 64.0f;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) pk[e] = pack_bf16x2(s[h2 * 64 + 2 * e], s[h2 * 64 + 2 * e + 1]);
        tc::tmem_st32(s_col + h2 * 32, pk);
      }
    }
    tc::tmem_wait_st();
    tc::fence_before_sync();
    // one arrive per warp (count 4): its lanes' TMEM stores are complete
    // (wait::st) and ordered before the elected arrive by __syncwarp
    __syncwarp();
    if ((tid & 31) == 0) mbar_arrive(&sm.p_full[j & 1]);
    __syncwarp();
  }

  // epilogue: (acc * f + g_acc) / (l * f + g_l), f re-bases acc and l on the final max.
  // Wait for every MMA of the tile on the single-phase mma_fin barrier: S(j+1)
  // is issued before P.V(j), so s_full(n-1) only implies that P.V(n-3) is
  // done, and P.V(n-2) and P.V(n-1) may still be running.
  warp_mbar_wait(&sm.mma_fin, 0u, p.err, kErrPvDone, abort_flag);
  tc::fence_after_sync();
  if (!staged) asm volatile("bar.sync 1, 128;" ::: "memory");
  const float f = ex2((m_ref - m_true) * sl2);
  const float denom = l * f + g_l;
  const float inv = denom == 0.f ? 0.f : 1.0f / denom;  // the reference's guard: 0 where the denominator is 0
  const int blk = half ? t.blk[1] : t.blk[0];
  const int token = blk * kBlock + (tid & 63);
  const bool write = (half == 0 || t.write1) && token < p.S;
  const float* oc = sm.outc[half];  // out_c * alpha (scalar alpha) or out_c
  const size_t out_row = ((size_t(t.b) * p.S + token) * p.H + t.h) * D;
  if (p.out_tma) {
    // bf16 output: stage the 128 x D tile in the (now idle) first key stage in
    // the TMA box layout (64 d per 128-byte row, 16-byte units swizzled with
    // the row, block B 8 KB after block A), then one thread writes it with
    // TMA stores (rows beyond S are clipped by the tensor map).
    uint8_t* stage = sm.k[0];
    const bool valid_row = token < p.S;
#pragma unroll 2
    for (int c = 0; c < D / 32; ++c) {
      uint32_t ro[32], rg[32];
      __syncwarp();
      tc::tmem_ld32(tmem + lanes + kSColO + c * 32, ro);
      tc::tmem_ld32(tmem + lanes + kSColG + c * 32, rg);
      tc::tmem_wait_ld();
      float o[32], x[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] = fmaf(__uint_as_float(ro[e]), f, __uint_as_float(rg[e])) * inv;
      if (valid_row && p.alpha_mode == ICSA_ALPHA_SCALAR) residual32_ca(oc, c * 32, o, x);
      else if (valid_row) residual32(p, t.b, token, t.h, oc, c * 32, o, x);
      else
#pragma unroll
        for (int e = 0; e < 32; ++e) x[e] = 0.f;
      uint8_t* row = stage + (c >> 1) * kChunkBytes + tid * 128;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint32_t unit = uint32_t((c & 1) * 4 + v);
        uint4 u;
        u.x = pack_bf16x2(x[v * 8 + 0], x[v * 8 + 1]);
        u.y = pack_bf16x2(x[v * 8 + 2], x[v * 8 + 3]);
        u.z = pack_bf16x2(x[v * 8 + 4], x[v * 8 + 5]);
        u.w = pack_bf16x2(x[v * 8 + 6], x[v * 8 + 7]);
        *reinterpret_cast<uint4*>(row + ((unit ^ uint32_t(tid & 7)) << 4)) = u;
      }
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (tid == 0) {
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        if (hb == 1 && !t.write1) continue;
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_store_4d(&maps.o, stage + c * kChunkBytes + hb * (kChunkBytes / 2), c * 64, t.h, t.blk[hb] * kBlock,
                       t.b);
      }
      bulk_commit();
      bulk_wait_read();
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    uint32_t ro[32], rg[32];
    __syncwarp();
    tc::tmem_ld32(tmem + lanes + kSColO + c * 32, ro);
    tc::tmem_ld32(tmem + lanes + kSColG + c * 32, rg);
    tc::tmem_wait_ld();
    float o[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      o[e] = fmaf(__uint_as_float(ro[e]), f, __uint_as_float(rg[e])) * inv;
    }
    if (!write) continue;
    if (p.alpha_mode == ICSA_ALPHA_SCALAR) {
      float x[32];
      residual32_ca(oc, c * 32, o, x);
      float* dst = reinterpret_cast<float*>(p.out) + out_row + c * 32;
      if (p.out_dtype == ICSA_BF16) {
        __nv_bfloat16* db = reinterpret_cast<__nv_bfloat16*>(p.out) + out_row + c * 32;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 u;
          u.x = pack_bf16x2(x[v * 8 + 0], x[v * 8 + 1]);
          u.y = pack_bf16x2(x[v * 8 + 2], x[v * 8 + 3]);
          u.z = pack_bf16x2(x[v * 8 + 4], x[v * 8 + 5]);
          u.w = pack_bf16x2(x[v * 8 + 6], x[v * 8 + 7]);
          reinterpret_cast<uint4*>(db)[v] = u;
        }
      } else {
#pragma unroll
        for (int v = 0; v < 8; ++v)
          reinterpret_cast<float4*>(dst)[v] = make_float4(x[v * 4], x[v * 4 + 1], x[v * 4 + 2], x[v * 4 + 3]);
      }
    } else {
      store_out32(p, t.b, token, t.h, oc, c * 32, o, out_row);
    }
  }
}

template <int D>
__global__ void __launch_bounds__(kSThreads, 1) sparse_kernel(const AttnParams p, const __grid_constant__ AttnMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  SSmem<D>& sm = *reinterpret_cast<SSmem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using C = SCfg<D>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const STile t = decode_sparse_tile(p, blockIdx.x);
  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&sm.k_full[i], 1);
      mbar_init(&sm.v_full[i], 1);
      mbar_init(&sm.v_empty[i], 1);
    }
    mbar_init(&sm.s_full[0], 1);
    mbar_init(&sm.s_full[1], 1);
    mbar_init(&sm.p_full[0], 4);
    mbar_init(&sm.p_full[1], 4);
    mbar_init(&sm.mma_fin, 1);
    sm.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kSMmaWarp) {
    tc::tmem_alloc(&sm.tmem_base, kSTmemCols);
    tc::tmem_relinquish();
  }
  if (warp == kSProducerWarp && lane == 0) {
    prefetch_tensormap(&maps.q);
    prefetch_tensormap(&maps.k);
    prefetch_tensormap(&maps.v);
    prefetch_tensormap(&maps.kc);
    prefetch_tensormap(&maps.vc);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  if (warp < 4) {
    sparse_softmax<D>(p, maps, t, sm, tmem);
  } else if (warp == kSProducerWarp) {
    if (lane == 0) {
      sparse_producer<D>(p, maps, t, sm);
      if (sm.abort_flag) {
        for (int j = max(0, t.n_steps - C::kStages); j < t.n_steps; ++j) {
          drain_wait(&sm.k_full[j % C::kStages], uint32_t(j / C::kStages) & 1u, p.err);
          drain_wait(&sm.v_full[j % C::kStages], uint32_t(j / C::kStages) & 1u, p.err);
        }
        drain_wait(&sm.q_full, 0, p.err);
      }
    }
  } else {
    sparse_mma<D>(p, t, sm, tmem);
    tc::mma_commit_elect(&sm.mma_fin);
    if (lane == 0) drain_wait(&sm.mma_fin, 0, p.err);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kSMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kSTmemCols);
  }
}

}  // namespace

cudaError_t launch_sparse_attention(const AttnParams& p, const AttnMaps& maps, int D, cudaStream_t stream) {
  const int ctas = p.B * p.H * p.sparse_tiles;
  if (ctas == 0) return cudaSuccess;
  if (D == 128) {
    const size_t smem = sizeof(SSmem<128>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(sparse_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    sparse_kernel<128><<<ctas, kSThreads, smem, stream>>>(p, maps);
  } else if (D == 64) {
    const size_t smem = sizeof(SSmem<64>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(sparse_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    sparse_kernel<64><<<ctas, kSThreads, smem, stream>>>(p, maps);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

ICSA_DEFINE_STICKY_ACCESSOR(sticky_status_sparse)

}  // namespace icsa
