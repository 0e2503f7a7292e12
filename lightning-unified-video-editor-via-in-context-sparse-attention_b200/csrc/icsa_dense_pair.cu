// Dense attention for the "flat" query blocks (the reference's
// flash_attn_func call, editing_sparse_attention.py:211-215, fused with the
// scatter and residual of :217-232), D = 128, on SM pairs.
//
// A cluster of two CTAs computes a 256-row query tile (four 64-token flat
// blocks): the leader issues M = 256 tcgen05 MMAs (cta_group::2), each CTA
// holds its own 128 query rows, half of every 128-row key tile (64 keys x
// 128 d) and half of every value tile (128 keys x 64 d).  Per CTA this reads
// 64 KB of operands from shared memory per 128 keys (plus 32 KB of TMA
// writes), under the 128 B/clk the tensor core can draw from it.
//
// TMEM (512 columns per CTA):
//   S at [0,128)                                  fp32 scores, lane = query row
//   P(j) in buffer j%2 at [128 + 64 (j%2), +64)   bf16 pairs (A operand of P.V)
//   O_w at [256 + 128 w, +128), w = 0, 1          fp32 accumulators
// Softmax warpgroup w owns the steps j with j % 2 == w, with P buffer w and
// its own accumulator O_w, exponent origin and row sum, so the two
// warpgroups never wait for each other; the epilogue brings O_0 and O_1 to
// a common origin.  Because P has its own columns, S(j+1) may overwrite S as
// soon as the softmax has copied S(j) to registers.  The tensor core's queue
// per step:  S(j+1) once softmax(j) has read S(j), then P.V(j-1) once P(j-1)
// is written.
//
// Roles per CTA (384 threads):
//   warps 0-3 / 4-7  softmax of the even / odd key steps, all 128 columns of
//                    every row (thread <-> TMEM lane <-> query row), each
//                    into its own accumulator;
//   warp 8           TMA producer (Q once, then the K and V rings);
//   warp 9           TMEM allocation; in the leader, the MMA issuer.
#include "icsa_attn_common.cuh"
#include "icsa_pair.cuh"

#include <utility>

namespace icsa {

namespace {

using namespace attn;

constexpr int kPThreads = 384;
constexpr int kPProducerWarp = 8;
constexpr int kPMmaWarp = 9;
constexpr int kPStages = 5;  // K/V ring: stage j % 5 holds this CTA's halves of K(j) and V(j)
constexpr int kPQBytes = 128 * 128 * 2;  // this CTA's 128 query rows, two 64-wide d chunks of 16 KB
constexpr int kPKBytes = 64 * 128 * 2;   // 64 key rows x 128 d, two d chunks of 8 KB
constexpr int kPVBytes = 128 * 64 * 2;   // 128 value rows x this CTA's 64 d
constexpr uint32_t kTmS = 0, kTmP = 128, kTmO = 256, kPTmemCols = 512;

struct __align__(1024) PSmem {
  uint8_t q[kPQBytes];
  uint8_t kv[kPStages][kPKBytes + kPVBytes];  // [K half | V half]
  float ocs[2][128];   // per query block: out_c * alpha (scalar alpha) or out_c
  float lsum[2][128];  // epilogue: partial row sums and their origins
  float lmax[2][128];
  uint64_t q_full;
  uint64_t kv_full[kPStages], kv_empty[kPStages];
  // [w]: barriers of softmax warpgroup w (steps j with j % 2 == w), so each
  // is consumed in phase order by one party
  uint64_t s_full[2], s_free[2], p_full[2];
  uint64_t pv_done[2];  // P.V(j) done, per P buffer j % 2
  uint64_t o_final;     // the last P.V done
  uint64_t mma_fin;
  uint32_t tmem_base;
  int abort_flag;
};

static_assert(sizeof(PSmem) + 1024 <= 232448, "pair kernel shared memory exceeds 227 KB");

struct PTile {
  int bh, b, h;
  int blk[2];    // query blocks of rows [0,64) and [64,128) of this CTA
  int write[2];  // 0 for a duplicate filling an incomplete group
  int n_steps;   // key steps of 128 rows
  uint32_t rank;
};

ICSA_DEV PTile decode_pair_tile(const AttnParams& p) {
  PTile t;
  t.rank = pair::cluster_rank();
  const int pr = blockIdx.x >> 1;
  const int groups = (p.num_flat + 3) / 4;
  t.bh = pr / groups;
  const int g = pr % groups;
  t.b = t.bh / p.H;
  t.h = t.bh % p.H;
  // flat blocks come first; no order table: query block r is block r
  const int* order = p.order ? p.order + size_t(t.bh) * p.NB : nullptr;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = 4 * g + 2 * int(t.rank) + i;
    t.write[i] = r < p.num_flat;
    const int rr = t.write[i] ? r : p.num_flat - 1;
    t.blk[i] = order ? order[rr] : rr;
  }
  t.n_steps = (p.nkv + 1) / 2;
  return t;
}

ICSA_DEV void pair_producer(const AttnParams& p, const AttnMaps& maps, const PTile& t, PSmem& sm) {
  volatile int* abort_flag = &sm.abort_flag;
  const bool leader = t.rank == 0;
  if (leader) mbar_arrive_expect_tx(&sm.q_full, 2 * kPQBytes);
  const uint32_t q_full = pair::mapa(&sm.q_full, 0);
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int half = 0; half < 2; ++half)
      pair::tma_load_4d(sm.q + c * kChunkBytes + half * (kChunkBytes / 2), &maps.q, q_full, c * 64, t.h,
                        t.blk[half] * kBlock, t.b);
  // no block table: KV block i starts at row 64 i
  const int* rows = p.kv_rows ? p.kv_rows + size_t(t.bh) * p.nkv : nullptr;
  for (int j = 0; j < t.n_steps; ++j) {
    const int s = j % kPStages;
    const uint32_t ph = uint32_t(j / kPStages) & 1u;
    const int r0 = rows ? rows[2 * j] : 2 * j * kBlock;
    const int r1 = (2 * j + 1 < p.nkv) ? (rows ? rows[2 * j + 1] : (2 * j + 1) * kBlock) : r0;  // missing half: masked by the softmax
    if (!mbar_wait(&sm.kv_empty[s], ph ^ 1u, p.err, kErrKEmpty, abort_flag)) return;
    if (leader) mbar_arrive_expect_tx(&sm.kv_full[s], 2 * (kPKBytes + kPVBytes));
    const uint32_t kv_full = pair::mapa(&sm.kv_full[s], 0);
    // keys: this CTA's 64 of the 128 (N split)
    const int rk = t.rank ? r1 : r0;
#pragma unroll
    for (int c = 0; c < 2; ++c)
      pair::tma_load_4d(sm.kv[s] + c * (kPKBytes / 2), &maps.k, kv_full, c * 64, t.h, rk, t.b);
    // values: all 128 keys, this CTA's 64 of the 128 d (N split)
    uint8_t* vdst = sm.kv[s] + kPKBytes;
    pair::tma_load_4d(vdst, &maps.v, kv_full, int(t.rank) * 64, t.h, r0, t.b);
    pair::tma_load_4d(vdst + kPVBytes / 2, &maps.v, kv_full, int(t.rank) * 64, t.h, r1, t.b);
  }
}

// S = Q K^T over d = 128: eight K = 16 steps; Q chunks are 16 KB apart, key
// chunks 8 KB apart; 32 bytes per step inside a 128-byte swizzled row.
template <int KK>
constexpr uint32_t kQOff = uint32_t(((KK >> 2) * kChunkBytes + (KK & 3) * 32) >> 4);
template <int KK>
constexpr uint32_t kKOff = uint32_t(((KK >> 2) * (kPKBytes / 2) + (KK & 3) * 32) >> 4);

template <int... KK>
ICSA_DEV void pair_issue_s_seq(uint64_t q_desc, uint64_t k_desc, uint32_t d_tmem, std::integer_sequence<int, KK...>) {
  constexpr uint32_t idesc = tc::make_idesc_bf16(256, 128, false, false);
  (pair::mma_ss_elect<kQOff<KK>, kKOff<KK>>(d_tmem, q_desc, k_desc, idesc, KK > 0 ? 1u : 0u), ...);
}

// O += P V over 128 keys: eight K = 16 steps; P advances 8 TMEM columns, V
// (MN-major, 128-byte rows of 64 d) advances 16 rows = 2048 bytes.
template <int... KK>
ICSA_DEV void pair_issue_pv_seq(uint64_t v_desc, uint32_t p_tmem, uint32_t o_tmem, uint32_t acc,
                                std::integer_sequence<int, KK...>) {
  constexpr uint32_t idesc = tc::make_idesc_bf16(256, 128, false, true);
  (pair::mma_ts_elect<uint32_t(KK * 8), uint32_t((KK * 16 * 128) >> 4)>(o_tmem, p_tmem, v_desc, idesc,
                                                                         (KK > 0) ? 1u : acc),
   ...);
}

// MMA issuer: all 32 lanes of warp 9 of the leader run this loop (waits are
// warp-uniform, one elected lane issues each instruction).
ICSA_DEV void pair_mma(const AttnParams& p, const PTile& t, PSmem& sm, uint32_t tmem) {
  volatile int* abort_flag = &sm.abort_flag;
  const int n = t.n_steps;
  const uint64_t qd = tc::make_sw128_desc(smem_u32(sm.q), 16, 1024);
  const uint64_t kd0 = tc::make_sw128_desc(smem_u32(sm.kv[0]), 16, 1024);
  const uint64_t vd0 = tc::make_sw128_desc(smem_u32(sm.kv[0] + kPKBytes), kPVBytes, 1024);
  constexpr uint64_t kKStep = uint64_t((kPKBytes + kPVBytes) >> 4), kVStep = kKStep;
  if (!warp_mbar_wait(&sm.q_full, 0, p.err, kErrQ, abort_flag)) return;

  auto issue_s = [&](int j) -> bool {
    const int s = j % kPStages;
    if (!warp_mbar_wait(&sm.kv_full[s], uint32_t(j / kPStages) & 1u, p.err, kErrKFull, abort_flag)) return false;
    tc::fence_after_sync();
    pair_issue_s_seq(qd, kd0 + uint64_t(s) * kKStep, tmem + kTmS, std::make_integer_sequence<int, 8>{});
    pair::commit_both_elect(&sm.s_full[j & 1]);
    return true;
  };
  auto issue_pv = [&](int j) -> bool {
    const int s = j % kPStages;
    if (!warp_mbar_wait(&sm.p_full[j & 1], uint32_t(j >> 1) & 1u, p.err, kErrPFull, abort_flag)) return false;
    tc::fence_after_sync();
    pair_issue_pv_seq(vd0 + uint64_t(s) * kVStep, tmem + kTmP + 64u * uint32_t(j & 1),
                      tmem + kTmO + 128u * uint32_t(j & 1), j >= 2 ? 1u : 0u, std::make_integer_sequence<int, 8>{});
    pair::commit_both_elect(&sm.pv_done[j & 1]);
    pair::commit_both_elect(&sm.kv_empty[s]);  // S(j) and P.V(j) have read stage s
    return true;
  };

  // The softmax warpgroups run half a step apart, so s_free(j) (early in
  // softmax j) and p_full(j-1) (end of softmax j-1) alternate:
  //   S(j+1) after s_free(j), P.V(j-1) after p_full(j-1).
  if (!issue_s(0)) return;
  for (int j = 0; j < n; ++j) {
    if (j + 1 < n) {
      if (!warp_mbar_wait(&sm.s_free[j & 1], uint32_t(j >> 1) & 1u, p.err, kErrSEmpty, abort_flag)) return;
      if (!issue_s(j + 1)) return;
    }
    if (j > 0 && !issue_pv(j - 1)) return;
  }
  if (!issue_pv(n - 1)) return;
  pair::commit_both_elect(&sm.o_final);
}

// Softmax: warpgroup w handles the key steps j with j % 2 == w, over all 128
// keys of the step (thread <-> TMEM lane <-> query row), into its own
// accumulator O_w with its own exponent origin m_w (raised lazily, when a
// step's maximum exceeds it by more than 2^8) and row sum l_w; the epilogue
// brings both to the larger origin.  The warpgroups therefore never wait
// for each other inside the loop.  Neither may leave the loop early (the
// epilogue's named barriers pair them): after a failed wait the abort flag
// is set, every later wait returns at once, the loop runs on over stale
// data, and the error code marks the result invalid.
ICSA_DEV void pair_softmax(const AttnParams& p, const AttnMaps& maps, const PTile& t, PSmem& sm, uint32_t tmem) {
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = warp >> 2;                 // this warpgroup's step parity
  const int row = threadIdx.x & 127;       // query row = TMEM lane
  const uint32_t lanes = uint32_t((warp & 3) * 32) << 16;
  const uint32_t s_base = tmem + lanes + kTmS;
  const uint32_t p_base = tmem + lanes + kTmP + 64u * uint32_t(w);
  const uint32_t o_base = tmem + lanes + kTmO;          // O_0 at +0, O_1 at +128
  const uint32_t o_own = o_base + 128u * uint32_t(w);
  // the residual term of the epilogue, one value per thread: block row >> 6,
  // feature (row & 63) + 64 w (read after the epilogue's barrier 14)
  {
    const int hb = row >> 6, d = (row & 63) + 64 * w;
    // no out_compress (plain attention): a zero residual term, x = bf16(o)
    const float cval = p.outc ? p.outc[(size_t(t.bh) * p.NB + (hb ? t.blk[1] : t.blk[0])) * 128 + d] : 0.f;
    sm.ocs[hb][d] = (p.alpha_mode == ICSA_ALPHA_SCALAR) ? ca_scalar(p, cval) : cval;
  }
  const uint32_t s_free = pair::mapa(&sm.s_free[w], 0);
  const uint32_t p_full = pair::mapa(&sm.p_full[w], 0);
  const float sl2 = p.scale_log2;
  const int n = t.n_steps;
  float m_w = -INFINITY, l_w = 0.f;  // this warpgroup's exponent origin and row sum

  for (int j = w; j < n; j += 2) {
    const uint32_t par = uint32_t(j >> 1) & 1u;
    warp_mbar_wait(&sm.s_full[w], par, p.err, kErrSFull, abort_flag);
    tc::fence_after_sync();
    float s[128];
    tmem_load_row128(s_base, s);
    // S may now be overwritten by S(j+1)
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) pair::arrive_cluster_relaxed(s_free);
    __syncwarp();

    const int hi = p.tkv - j * 128;  // extended-KV rows beyond tkv are not keys
    if (hi < 128) {
#pragma unroll
      for (int c = 0; c < 128; ++c)
        if (c >= hi) s[c] = -INFINITY;
    }
    const float mx = max128(s);
    const bool need = (mx - m_w) * sl2 > kRescaleThreshold;
    const float m_ref = need ? mx : m_w;
    const float alpha = (need && m_w != -INFINITY) ? ex2((m_w - m_ref) * sl2) : 1.f;
    if (need) {
      l_w = (m_w == -INFINITY) ? 0.f : l_w * alpha;
      m_w = m_ref;
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
    }
    l_w += (a0 + a1) + (a2 + a3);
    // P buffer w and O_w were last used by P.V(j-2); the phase before it on
    // its barrier, P.V(j-4), was issued before S(j-1) and has completed
    if (j >= 2) {
      warp_mbar_wait(&sm.pv_done[w], uint32_t((j - 2) >> 1) & 1u, p.err, kErrPvDone, abort_flag);
      tc::fence_after_sync();
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tc::tmem_ld32(o_own + 32u * uint32_t(c), r);
          tc::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
          tc::tmem_st32(o_own + 32u * uint32_t(c), r);
        }
      }
    }
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      uint32_t pk[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) pk[e] = pack_bf16x2(s[64 * h2 + 2 * e], s[64 * h2 + 2 * e + 1]);
      tc::tmem_st32(p_base + uint32_t(h2) * 32u, pk);
    }
    tc::tmem_wait_st();
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) pair::arrive_cluster_relaxed(p_full);
    __syncwarp();
  }

  // epilogue: both accumulators and row sums to the larger origin; this
  // warpgroup writes features [64w, 64w + 64) of its row
  warp_mbar_wait(&sm.o_final, 0, p.err, kErrPvDone, abort_flag);
  tc::fence_after_sync();
  sm.lsum[w][row] = l_w;
  sm.lmax[w][row] = m_w;
  pair::named_sync(9u + uint32_t(warp & 3), 64);
  const float m0 = sm.lmax[0][row], m1 = sm.lmax[1][row];
  const float m_fin = fmaxf(m0, m1);
  const bool has1 = n >= 2;  // O_1 holds data only when warpgroup 1 had steps
  const float f0 = (m0 == -INFINITY) ? 0.f : ex2((m0 - m_fin) * sl2);
  const float f1 = (!has1 || m1 == -INFINITY) ? 0.f : ex2((m1 - m_fin) * sl2);
  const float lt = sm.lsum[0][row] * f0 + (has1 ? sm.lsum[1][row] * f1 : 0.f);
  const float inv = lt == 0.f ? 0.f : 1.0f / lt;
  const int hb = row >> 6;
  const int blk = hb ? t.blk[1] : t.blk[0];  // (no dynamic indexing: keeps the tile in registers)
  const int token = blk * kBlock + (row & 63);
  const bool valid_row = token < p.S;
  const bool write = (hb ? t.write[1] : t.write[0]) && valid_row;
  pair::named_sync(14, 256);  // sm.ocs complete
  const float* oc = sm.ocs[hb];
  const bool scalar = p.alpha_mode == ICSA_ALPHA_SCALAR;
  const size_t out_row = ((size_t(t.b) * p.S + token) * p.H + t.h) * 128;
  if (p.out_tma) {
    // bf16 output: stage this CTA's 128 x 128 tile in the idle first K/V stage
    // in the TMA box layout (64 d per 128-byte row, 16-byte units swizzled
    // with the row, block B 8 KB after block A; warpgroup w fills d chunk w),
    // then one thread writes it with TMA stores (rows beyond S are clipped).
    uint8_t* stage = sm.kv[0];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
      __syncwarp();
      tc::tmem_ld32(o_base + 64u * uint32_t(w) + 32u * uint32_t(c), r);
      uint32_t r1[32];
      if (has1) tc::tmem_ld32(o_base + 128u + 64u * uint32_t(w) + 32u * uint32_t(c), r1);
      tc::tmem_wait_ld();
      float o[32], x[32];
#pragma unroll
      for (int e = 0; e < 32; ++e)
        o[e] = (__uint_as_float(r[e]) * f0 + (has1 ? __uint_as_float(r1[e]) * f1 : 0.f)) * inv;
      if (valid_row && scalar) residual32_ca(oc, 64 * w + 32 * c, o, x);
      else if (valid_row) residual32(p, t.b, token, t.h, oc, 64 * w + 32 * c, o, x);
      else
#pragma unroll
        for (int e = 0; e < 32; ++e) x[e] = 0.f;
      uint8_t* rp = stage + w * kChunkBytes + row * 128;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint32_t unit = uint32_t(c * 4 + v);
        uint4 u;
        u.x = pack_bf16x2(x[v * 8 + 0], x[v * 8 + 1]);
        u.y = pack_bf16x2(x[v * 8 + 2], x[v * 8 + 3]);
        u.z = pack_bf16x2(x[v * 8 + 4], x[v * 8 + 5]);
        u.w = pack_bf16x2(x[v * 8 + 6], x[v * 8 + 7]);
        *reinterpret_cast<uint4*>(rp + ((unit ^ uint32_t(row & 7)) << 4)) = u;
      }
    }
    fence_proxy_async_smem();
    pair::named_sync(15, 256);
    if (threadIdx.x == 0) {
#pragma unroll
      for (int b2 = 0; b2 < 2; ++b2) {
        if (!t.write[b2]) continue;
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tma_store_4d(&maps.o, stage + c * kChunkBytes + b2 * (kChunkBytes / 2), c * 64, t.h, t.blk[b2] * kBlock,
                       t.b);
      }
      bulk_commit();
      bulk_wait_read();
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint32_t r[32];
    __syncwarp();
    tc::tmem_ld32(o_base + 64u * uint32_t(w) + 32u * uint32_t(c), r);
    uint32_t r1[32];
    if (has1) tc::tmem_ld32(o_base + 128u + 64u * uint32_t(w) + 32u * uint32_t(c), r1);
    tc::tmem_wait_ld();
    float o[32];
#pragma unroll
    for (int e = 0; e < 32; ++e)
      o[e] = (__uint_as_float(r[e]) * f0 + (has1 ? __uint_as_float(r1[e]) * f1 : 0.f)) * inv;
    if (!write) continue;
    if (scalar) {
      float x[32];
      residual32_ca(oc, 64 * w + 32 * c, o, x);
      if (p.out_dtype == ICSA_BF16) {
        __nv_bfloat16* db = reinterpret_cast<__nv_bfloat16*>(p.out) + out_row + 64 * w + 32 * c;
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
        float* df = reinterpret_cast<float*>(p.out) + out_row + 64 * w + 32 * c;
#pragma unroll
        for (int v = 0; v < 8; ++v)
          reinterpret_cast<float4*>(df)[v] = make_float4(x[v * 4], x[v * 4 + 1], x[v * 4 + 2], x[v * 4 + 3]);
      }
    } else {
      store_out32(p, t.b, token, t.h, oc, 64 * w + 32 * c, o, out_row);
    }
  }
}
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    dense_pair_kernel(const AttnParams p, const __grid_constant__ AttnMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  PSmem& sm = *reinterpret_cast<PSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const PTile t = decode_pair_tile(p);

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], 8);  // one arrival per warp of the step's warpgroup, both CTAs
      mbar_init(&sm.p_full[i], 8);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&sm.pv_done[i], 1);
    mbar_init(&sm.o_final, 1);
    mbar_init(&sm.mma_fin, 1);
    sm.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kPMmaWarp) {
    pair::tmem_alloc(&sm.tmem_base, kPTmemCols);
    pair::tmem_relinquish();
  }
  if (warp == kPProducerWarp && lane == 0) {
    prefetch_tensormap(&maps.q);
    prefetch_tensormap(&maps.k);
    prefetch_tensormap(&maps.v);
  }
  tc::fence_before_sync();
  pair::cluster_sync();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  // Register split: 384 threads launch with 168 registers each; warpgroup 2
  // (producer, MMA issuer, two idle warps) gives registers back so that the
  // softmax warpgroups can hold a whole 128-column row:
  // 256 x 216 + 128 x 72 = 384 x 168.  setmaxnreg is executed by every warp of
  // a warpgroup.
  if (warp < 8) {
    tc::reg_alloc<216>();
    pair_softmax(p, maps, t, sm, tmem);
  } else {
    tc::reg_dealloc<72>();
  }
  if (warp == kPProducerWarp) {
    if (lane == 0) {
      pair_producer(p, maps, t, sm);
      if (sm.abort_flag && t.rank == 0) {
        // the leader's full barriers count the bytes of both CTAs: let every
        // copy still in flight land before either CTA releases its memory
        for (int j = max(0, t.n_steps - kPStages); j < t.n_steps; ++j) {
          drain_wait(&sm.kv_full[j % kPStages], uint32_t(j / kPStages) & 1u, p.err);
        }
        drain_wait(&sm.q_full, 0, p.err);
      }
    }
  } else if (warp == kPMmaWarp) {
    if (t.rank == 0) {
      pair_mma(p, t, sm, tmem);
      pair::commit_both_elect(&sm.mma_fin);
      if (lane == 0) drain_wait(&sm.mma_fin, 0, p.err);
    }
  }
  __syncwarp();
  tc::fence_before_sync();
  pair::cluster_sync();
  if (warp == kPMmaWarp) {
    tc::fence_after_sync();
    pair::tmem_dealloc(tmem, kPTmemCols);
  }
}

}  // namespace

cudaError_t launch_dense_pair_attention(const AttnParams& p, const AttnMaps& maps, cudaStream_t stream) {
  const int pairs = p.B * p.H * ((p.num_flat + 3) / 4);
  if (pairs == 0) return cudaSuccess;
  const size_t smem = sizeof(PSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(dense_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dense_pair_kernel<<<2 * pairs, kPThreads, smem, stream>>>(p, maps);
  return cudaGetLastError();
}

ICSA_DEFINE_STICKY_ACCESSOR(sticky_status_dense_pair)

}  // namespace icsa
