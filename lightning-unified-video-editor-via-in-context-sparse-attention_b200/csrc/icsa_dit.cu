// Fused elementwise stages of one Wan 2.2 DiT block: the HBM passes between
// the block's GEMMs (reference model.py:152-170 and :248-265).
//
// All three kernels are bandwidth-bound row passes.  One CTA of 128 threads
// owns one row of the model width C (5120 for the A14B model); every thread
// holds KC = ceil(C / 1024) chunks of 8 consecutive columns in registers, at
// columns (k * 128 + tid) * 8, so a warp's loads cover 512 contiguous bytes of
// bf16 (1 KB of f32) and the row is read exactly once.  Row statistics are two
// block reductions over those registers (mean, then the centred second moment
// for LayerNorm; the mean square for RMSNorm).
//
// Rounding follows the reference's dtype flow under CUDA autocast (bf16
// GEMMs, f32 residual stream):
//   * WanLayerNorm (model.py:116-121) normalises in f32 and casts back to the
//     residual stream's dtype; `* (1 + e[1]) + e[0]` are two f32 ops, and the
//     next Linear casts to bf16 (model.py:256, :263);
//   * WanRMSNorm (model.py:102-113): bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w);
//   * rope_apply (model.py:69-95) multiplies in complex128 and returns f32;
//   * alpha_1 (model.py:162): sigmoid, - 0.5 and * 0.5 each rounded to bf16;
//   * `x + y * e` (model.py:259, :265): f32 product, then f32 sum.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <type_traits>

#include "icsa_kernels.cuh"
#include "icsa_dit.h"

extern "C" void icsa_set_last_error(const char* msg);

namespace icsa {
namespace {

constexpr int kRowThreads = 128;
constexpr int kMaxChunks = 8;  // C <= 8192

int dit_fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int dit_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  icsa_set_last_error(buf);
  return code;
}

int dit_launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return dit_fail(ICSA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ICSA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

ICSA_DEV float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const float t = (red[0] + red[1]) + (red[2] + red[3]);
  __syncthreads();
  return t;
}

ICSA_DEV void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

ICSA_DEV void load8(const float* p, float (&f)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

ICSA_DEV void store8_bf16(void* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

ICSA_DEV void store8_f32(void* p, const float (&f)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// ---------------------------------------------------------------------------
// Modulated LayerNorm
// ---------------------------------------------------------------------------
struct ModNormArgs {
  const void* x;
  int64_t ldx;
  int rows, C, rows_per_batch;
  const float* scale;
  int64_t scale_bs;
  const float* shift;
  int64_t shift_bs;
  float eps;
  int round_norm;
  __nv_bfloat16* out;
};

template <int KC, typename TX>
__global__ void __launch_bounds__(kRowThreads) modulated_norm_kernel(ModNormArgs a) {
  __shared__ float red[4];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const TX* x = reinterpret_cast<const TX*>(a.x) + size_t(row) * a.ldx;
  float v[KC][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < KC; ++k) {
    const int col = (k * kRowThreads + tid) * 8;
    if (col < a.C) {
      load8(x + col, v[k]);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[k][i];
    }
  }
  const float mean = block_sum(s, red) / float(a.C);
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < KC; ++k) {
    const int col = (k * kRowThreads + tid) * 8;
    if (col < a.C) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[k][i] - mean;
        q = fmaf(d, d, q);
      }
    }
  }
  const float rstd = rsqrtf(block_sum(q, red) / float(a.C) + a.eps);
  const int b = row / a.rows_per_batch;
  const float* sc = a.scale + size_t(b) * a.scale_bs;
  const float* sh = a.shift + size_t(b) * a.shift_bs;
#pragma unroll
  for (int k = 0; k < KC; ++k) {
    const int col = (k * kRowThreads + tid) * 8;
    if (col < a.C) {
      float g[8], h[8], y[8];
      load8(sc + col, g);
      load8(sh + col, h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float n = (v[k][i] - mean) * rstd;
        if (a.round_norm) n = bf16_round(n);
        y[i] = __fadd_rn(__fmul_rn(n, g[i]), h[i]);
      }
      store8_bf16(a.out + size_t(row) * a.C + col, y);
    }
  }
}

// ---------------------------------------------------------------------------
// RMSNorm + rotary embedding + layout change (+ gate)
// ---------------------------------------------------------------------------
struct NormRopeArgs {
  int rows, C, D, rows_per_batch, token_offset;
  int64_t ld;
  float eps;
  const __nv_bfloat16* src[3];
  const __nv_bfloat16* w[3];
  int rope[3];
  void* dst[3];
  int dst_f32[3];
  int hp;
  int64_t sb, sg, st;
  const double2* table;
  int positions;
  const int4* token_pos;
  int token_count;
  int split1, split2;
  const __nv_bfloat16* gate_src;
  __nv_bfloat16* gate_dst;
};

template <int KC>
__global__ void __launch_bounds__(kRowThreads) norm_rope_kernel(NormRopeArgs a) {
  __shared__ float red[4];
  const int row = blockIdx.x;
  const int j = blockIdx.y;
  const int tid = threadIdx.x;
  const __nv_bfloat16* src = a.src[j] + size_t(row) * a.ld;
  const __nv_bfloat16* w = a.w[j];
  float v[KC][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < KC; ++k) {
    const int col = (k * kRowThreads + tid) * 8;
    if (col < a.C) {
      load8(src + col, v[k]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[k][i], v[k][i], ss);
    }
  }
  float rs = 1.f;
  if (w != nullptr) rs = rsqrtf(block_sum(ss, red) / float(a.C) + a.eps);

  const int b = row / a.rows_per_batch;
  const int t_local = row - b * a.rows_per_batch;
  int4 pos = make_int4(0, 0, 0, 0);
  if (a.rope[j]) {
    const int t = min(max(a.token_offset + t_local, 0), a.token_count - 1);
    pos = a.token_pos[t];
    pos.x = min(max(pos.x, 0), a.positions - 1);
    pos.y = min(max(pos.y, 0), a.positions - 1);
    pos.z = min(max(pos.z, 0), a.positions - 1);
  }
  const int half = a.D >> 1;
#pragma unroll
  for (int k = 0; k < KC; ++k) {
    const int col = (k * kRowThreads + tid) * 8;
    if (col < a.C) {
      float n[8];
      if (w != nullptr) {
        float wf[8];
        load8(w + col, wf);
#pragma unroll
        for (int i = 0; i < 8; ++i) n[i] = bf16_round(bf16_round(v[k][i] * rs) * wf[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) n[i] = v[k][i];
      }
      const int h = col / a.D;
      const int d = col - h * a.D;
      if (a.rope[j] && pos.w != 0) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const int pair = (d + i) >> 1;
          const int p = pair < a.split1 ? pos.x : (pair < a.split2 ? pos.y : pos.z);
          const double2 cs = a.table[size_t(p) * half + pair];
          const double re = double(n[i]), im = double(n[i + 1]);
          n[i] = float(re * cs.x - im * cs.y);
          n[i + 1] = float(re * cs.y + im * cs.x);
        }
      }
      const int g = h / a.hp;
      const int64_t off = b * a.sb + g * a.sg + t_local * a.st + int64_t(h - g * a.hp) * a.D + d;
      if (a.dst_f32[j])
        store8_f32(reinterpret_cast<float*>(a.dst[j]) + off, n);
      else
        store8_bf16(reinterpret_cast<__nv_bfloat16*>(a.dst[j]) + off, n);
    }
  }
  if (j == 0 && tid == 0 && a.gate_src != nullptr) {
    const float x = __bfloat162float(a.gate_src[size_t(row) * a.ld]);
    const float sg = bf16_round(1.f / (1.f + expf(-x)));
    const float c = bf16_round(sg - 0.5f);
    a.gate_dst[row] = __float2bfloat16_rn(c * 0.5f);
  }
}

// ---------------------------------------------------------------------------
// RMSNorm + RoPE with the 64-token block pooling of the result (the producer
// side of the attention's pooling stage), in two passes:
//   row_rms_kernel        rs = rsqrt(mean(x^2) + eps) per row, with the same
//                         arithmetic (and so the same bits) as norm_rope_kernel;
//   norm_rope_pool_kernel one CTA per (64-token block, 512-column slab,
//                         vector): each thread owns 8 columns, walks the
//                         block's 64 rows in order, writes the normalised and
//                         rotated values as bf16 into the exchange layout and
//                         sums their float32 values, so the block mean is the
//                         one the attention's pool_kernel takes of the float32
//                         result (rows summed in order, / 64, rounded to bf16
//                         values when the compressed attention runs in bf16).
// The float32 vectors themselves never reach HBM.
// ---------------------------------------------------------------------------
struct RowRmsArgs {
  const __nv_bfloat16* src[3];
  float* rs[3];
  int rows, C;
  int64_t ld;
  float eps;
};

template <int KC>
__global__ void __launch_bounds__(kRowThreads) row_rms_kernel(RowRmsArgs a) {
  __shared__ float red[4];
  const int row = blockIdx.x;
  const int j = blockIdx.y;
  // selects instead of a dynamic index, which would copy the arrays to local memory
  float* rs_out = j == 0 ? a.rs[0] : (j == 1 ? a.rs[1] : a.rs[2]);
  if (rs_out == nullptr) return;
  const int tid = threadIdx.x;
  const __nv_bfloat16* src = (j == 0 ? a.src[0] : (j == 1 ? a.src[1] : a.src[2])) + size_t(row) * a.ld;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < KC; ++k) {
    const int col = (k * kRowThreads + tid) * 8;
    if (col < a.C) {
      float v[8];
      load8(src + col, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
    }
  }
  const float rs = rsqrtf(block_sum(ss, red) / float(a.C) + a.eps);
  if (tid == 0) rs_out[row] = rs;
}

constexpr int kPoolSlab = 512;              // columns per CTA
constexpr int kPoolThreadsDit = kPoolSlab / 8;

struct RopePoolArgs {
  NormRopeArgs n;            // sources, weights, rope, bf16 destinations and their strides
  const float* rs[3];        // per-row rsqrt factors of the normalised vectors
  float* mean[3];            // f32 block means, or nullptr
  __nv_bfloat16* sum[3];     // bf16 block sums of the bf16 outputs, or nullptr
  int bf16_mean[3];          // mean of the bf16 outputs in bf16 arithmetic
  int64_t mb, mg;            // mean / sum offset of (b, g): b*mb + g*mg + (hl*nbl + blk)*D + d
  int nbl;                   // 64-token blocks per batch element
  int round_mean;
};

__global__ void __launch_bounds__(kPoolThreadsDit) norm_rope_pool_kernel(RopePoolArgs pa) {
  const NormRopeArgs& a = pa.n;
  const int j = blockIdx.z;
  const int b = blockIdx.x / pa.nbl;
  const int blk = blockIdx.x - b * pa.nbl;
  const int col = blockIdx.y * kPoolSlab + threadIdx.x * 8;
  const __nv_bfloat16* w = a.w[j];
  const float* rs = pa.rs[j];
  // gate alpha_1 of the block's rows: one thread of the first vector's first slab
  if (j == 0 && blockIdx.y == 0 && threadIdx.x < 64 && a.gate_src != nullptr) {
    const int row = b * a.rows_per_batch + blk * 64 + threadIdx.x;
    const float x = __bfloat162float(a.gate_src[size_t(row) * a.ld]);
    const float sg = bf16_round(1.f / (1.f + expf(-x)));
    const float c = bf16_round(sg - 0.5f);
    a.gate_dst[row] = __float2bfloat16_rn(c * 0.5f);
  }
  if (col >= a.C) return;
  const int h = col / a.D;
  const int d = col - h * a.D;
  const int g = h / a.hp;
  const int hl = h - g * a.hp;
  const int half = a.D >> 1;
  float wf[8];
  if (w != nullptr) load8(w + col, wf);
  float sum[8], sum_bf[8];  // of the float32 results / of their bf16 roundings
#pragma unroll
  for (int i = 0; i < 8; ++i) sum[i] = sum_bf[i] = 0.f;
  // selects instead of dynamic indexing of the parameter arrays
  float* mean_out = j == 0 ? pa.mean[0] : (j == 1 ? pa.mean[1] : pa.mean[2]);
  __nv_bfloat16* sum_out = j == 0 ? pa.sum[0] : (j == 1 ? pa.sum[1] : pa.sum[2]);
  const bool bf16_mean = (j == 0 ? pa.bf16_mean[0] : (j == 1 ? pa.bf16_mean[1] : pa.bf16_mean[2])) != 0;
  const bool pool = mean_out != nullptr || sum_out != nullptr;
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.dst[j]) + b * a.sb + g * a.sg + int64_t(hl) * a.D + d;
#pragma unroll 4
  for (int r = 0; r < 64; ++r) {
    const int t_local = blk * 64 + r;
    const int row = b * a.rows_per_batch + t_local;
    float n[8];
    load8(a.src[j] + size_t(row) * a.ld + col, n);
    if (w != nullptr) {
      const float f = rs[row];
#pragma unroll
      for (int i = 0; i < 8; ++i) n[i] = bf16_round(bf16_round(n[i] * f) * wf[i]);
    }
    if (a.rope[j]) {
      const int t = min(max(a.token_offset + t_local, 0), a.token_count - 1);
      int4 pos = a.token_pos[t];
      if (pos.w != 0) {
        pos.x = min(max(pos.x, 0), a.positions - 1);
        pos.y = min(max(pos.y, 0), a.positions - 1);
        pos.z = min(max(pos.z, 0), a.positions - 1);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const int pair = (d + i) >> 1;
          const int p = pair < a.split1 ? pos.x : (pair < a.split2 ? pos.y : pos.z);
          const double2 cs = a.table[size_t(p) * half + pair];
          const double re = double(n[i]), im = double(n[i + 1]);
          n[i] = float(re * cs.x - im * cs.y);
          n[i + 1] = float(re * cs.y + im * cs.x);
        }
      }
    }
    store8_bf16(dst + int64_t(t_local) * a.st, n);
    if (pool) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sum[i] += n[i];
        sum_bf[i] += bf16_round(n[i]);
      }
    }
  }
  if (pool) {
    const int64_t o = b * pa.mb + g * pa.mg + (int64_t(hl) * pa.nbl + blk) * a.D + d;
    if (mean_out != nullptr) {
      float mean[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (bf16_mean) {
          mean[i] = bf16_round(bf16_round(sum_bf[i]) / 64.f);
        } else {
          mean[i] = sum[i] / 64.f;
          if (pa.round_mean) mean[i] = bf16_round(mean[i]);
        }
      }
      store8_f32(mean_out + o, mean);
    }
    if (sum_out != nullptr) store8_bf16(sum_out + o, sum_bf);
  }
}

// ---------------------------------------------------------------------------
// Gated residual
// ---------------------------------------------------------------------------
struct GateArgs {
  float* x;
  const __nv_bfloat16* y;
  int64_t ldy;
  int rows, C, rows_per_batch;
  const float* gate;
  int64_t gate_bs;
};

__global__ void __launch_bounds__(256) gated_residual_kernel(GateArgs a) {
  const int cols8 = a.C >> 3;
  const int64_t n8 = int64_t(a.rows) * cols8;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const int row = int(i / cols8);
    const int col = int(i - int64_t(row) * cols8) * 8;
    float* xp = a.x + size_t(row) * a.C + col;
    float x[8], y[8];
    load8(xp, x);
    load8(a.y + size_t(row) * a.ldy + col, y);
    if (a.gate != nullptr) {
      float g[8];
      load8(a.gate + size_t(row / a.rows_per_batch) * a.gate_bs + col, g);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __fadd_rn(x[e], __fmul_rn(y[e], g[e]));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __fadd_rn(x[e], y[e]);
    }
    store8_f32(xp, x);
  }
}

template <typename F>
cudaError_t dispatch_chunks(int C, F&& f) {
  switch ((C + kRowThreads * 8 - 1) / (kRowThreads * 8)) {
    case 1: return f(std::integral_constant<int, 1>{});
    case 2: return f(std::integral_constant<int, 2>{});
    case 3: return f(std::integral_constant<int, 3>{});
    case 4: return f(std::integral_constant<int, 4>{});
    case 5: return f(std::integral_constant<int, 5>{});
    case 6: return f(std::integral_constant<int, 6>{});
    case 7: return f(std::integral_constant<int, 7>{});
    default: return f(std::integral_constant<int, 8>{});
  }
}

}  // namespace
}  // namespace icsa

namespace icsa {
namespace {
// Checks a descriptor and fills the kernel arguments.
int norm_rope_args(const icsa_dit_norm_rope_desc* d, NormRopeArgs& a) {
  if (d == nullptr) return dit_fail(ICSA_ERR_INVALID, "norm_rope: descriptor is NULL");
  if (d->count < 1 || d->count > 3) return dit_fail(ICSA_ERR_INVALID, "norm_rope: count=%d must be 1..3", d->count);
  if (d->rows < 0 || d->D < 8 || d->D % 8 || d->C < d->D || d->C % d->D || d->C > kMaxChunks * kRowThreads * 8 ||
      d->ld < d->C || d->ld % 8 || d->rows_per_batch < 1)
    return dit_fail(ICSA_ERR_INVALID, "norm_rope: rows=%d C=%d D=%d ld=%lld rows_per_batch=%d", d->rows, d->C, d->D,
                    (long long)d->ld, d->rows_per_batch);
  const int heads = d->C / d->D;
  if (d->heads_per_group < 1 || heads % d->heads_per_group)
    return dit_fail(ICSA_ERR_INVALID, "norm_rope: heads_per_group=%d must divide %d heads", d->heads_per_group, heads);
  if (d->dst_batch_stride % 8 || d->dst_group_stride % 8 || d->dst_token_stride % 8 || d->dst_batch_stride < 0 ||
      d->dst_group_stride < 0 || d->dst_token_stride < 0)
    return dit_fail(ICSA_ERR_INVALID, "norm_rope: destination strides must be non-negative multiples of 8");
  a = NormRopeArgs{};
  a.rows = d->rows; a.C = d->C; a.D = d->D; a.rows_per_batch = d->rows_per_batch; a.token_offset = d->token_offset;
  a.ld = d->ld; a.eps = d->eps; a.hp = d->heads_per_group;
  a.sb = d->dst_batch_stride; a.sg = d->dst_group_stride; a.st = d->dst_token_stride;
  bool any_rope = false;
  for (int j = 0; j < d->count; ++j) {
    if (d->src[j] == nullptr || d->dst[j] == nullptr)
      return dit_fail(ICSA_ERR_INVALID, "norm_rope: vector %d has a NULL source or destination", j);
    if (!aligned16(d->src[j]) || !aligned16(d->dst[j]) || (d->norm_weight[j] && !aligned16(d->norm_weight[j])))
      return dit_fail(ICSA_ERR_INVALID, "norm_rope: vector %d buffers must be 16-byte aligned", j);
    if (d->dst_dtype[j] != ICSA_BF16 && d->dst_dtype[j] != ICSA_F32)
      return dit_fail(ICSA_ERR_INVALID, "norm_rope: vector %d has a bad destination dtype", j);
    a.src[j] = reinterpret_cast<const __nv_bfloat16*>(d->src[j]);
    a.w[j] = reinterpret_cast<const __nv_bfloat16*>(d->norm_weight[j]);
    a.rope[j] = d->rope[j] ? 1 : 0;
    a.dst[j] = d->dst[j];
    a.dst_f32[j] = d->dst_dtype[j] == ICSA_F32;
    any_rope = any_rope || a.rope[j];
  }
  if (any_rope) {
    const int half = d->D / 2;
    if (d->rope_table == nullptr || d->token_pos == nullptr || d->rope_positions < 1 || d->token_count < 1)
      return dit_fail(ICSA_ERR_INVALID, "norm_rope: rotary embedding needs a table and token positions");
    if (d->rope_split1 < 0 || d->rope_split1 > d->rope_split2 || d->rope_split2 > half)
      return dit_fail(ICSA_ERR_INVALID, "norm_rope: splits %d, %d must satisfy 0 <= s1 <= s2 <= D/2", d->rope_split1,
                      d->rope_split2);
    if (!aligned16(d->rope_table) || !aligned16(d->token_pos))
      return dit_fail(ICSA_ERR_INVALID, "norm_rope: table and positions must be 16-byte aligned");
    a.table = reinterpret_cast<const double2*>(d->rope_table);
    a.positions = d->rope_positions;
    a.token_pos = reinterpret_cast<const int4*>(d->token_pos);
    a.token_count = d->token_count;
    a.split1 = d->rope_split1;
    a.split2 = d->rope_split2;
  }
  if (d->gate_src != nullptr) {
    if (d->gate_dst == nullptr) return dit_fail(ICSA_ERR_INVALID, "norm_rope: gate_dst is NULL");
    a.gate_src = reinterpret_cast<const __nv_bfloat16*>(d->gate_src);
    a.gate_dst = reinterpret_cast<__nv_bfloat16*>(d->gate_dst);
  }
  return ICSA_OK;
}
}  // namespace
}  // namespace icsa

using namespace icsa;

extern "C" {

int icsa_dit_modulated_norm(const void* x, int x_dtype, int64_t ldx, int rows, int C, int rows_per_batch,
                            const float* scale, int64_t scale_batch_stride, const float* shift,
                            int64_t shift_batch_stride, float eps, int round_norm_bf16, void* out,
                            cudaStream_t stream) {
  if (x == nullptr || scale == nullptr || shift == nullptr || out == nullptr)
    return dit_fail(ICSA_ERR_INVALID, "modulated_norm: NULL buffer");
  if (x_dtype != ICSA_BF16 && x_dtype != ICSA_F32) return dit_fail(ICSA_ERR_INVALID, "modulated_norm: bad x dtype");
  if (rows < 0 || C < 8 || C % 8 || C > kMaxChunks * kRowThreads * 8 || rows_per_batch < 1 || ldx < C || ldx % 8)
    return dit_fail(ICSA_ERR_INVALID, "modulated_norm: rows=%d C=%d ldx=%lld rows_per_batch=%d", rows, C,
                    (long long)ldx, rows_per_batch);
  if (scale_batch_stride < 0 || shift_batch_stride < 0 || scale_batch_stride % 4 || shift_batch_stride % 4)
    return dit_fail(ICSA_ERR_INVALID, "modulated_norm: batch strides must be non-negative multiples of 4");
  if (!aligned16(x) || !aligned16(scale) || !aligned16(shift) || !aligned16(out))
    return dit_fail(ICSA_ERR_INVALID, "modulated_norm: buffers must be 16-byte aligned");
  if (rows == 0) return ICSA_OK;
  ModNormArgs a{x, ldx, rows, C, rows_per_batch, scale, scale_batch_stride, shift, shift_batch_stride, eps,
                round_norm_bf16 ? 1 : 0, reinterpret_cast<__nv_bfloat16*>(out)};
  dispatch_chunks(C, [&](auto kc) {
    constexpr int KC = decltype(kc)::value;
    if (x_dtype == ICSA_F32)
      modulated_norm_kernel<KC, float><<<rows, kRowThreads, 0, stream>>>(a);
    else
      modulated_norm_kernel<KC, __nv_bfloat16><<<rows, kRowThreads, 0, stream>>>(a);
    return cudaSuccess;
  });
  return dit_launch_status("modulated_norm launch");
}

int icsa_dit_norm_rope(const icsa_dit_norm_rope_desc* d, cudaStream_t stream) {
  NormRopeArgs a{};
  const int rc = norm_rope_args(d, a);
  if (rc != ICSA_OK) return rc;
  if (d->rows == 0) return ICSA_OK;
  const dim3 grid(d->rows, d->count);
  dispatch_chunks(d->C, [&](auto kc) {
    constexpr int KC = decltype(kc)::value;
    norm_rope_kernel<KC><<<grid, kRowThreads, 0, stream>>>(a);
    return cudaSuccess;
  });
  return dit_launch_status("norm_rope launch");
}

int icsa_dit_norm_rope_pool(const icsa_dit_norm_rope_pool_desc* pd, cudaStream_t stream) {
  if (pd == nullptr) return dit_fail(ICSA_ERR_INVALID, "norm_rope_pool: descriptor is NULL");
  const icsa_dit_norm_rope_desc* d = &pd->base;
  NormRopeArgs a{};
  int rc = norm_rope_args(d, a);
  if (rc != ICSA_OK) return rc;
  if (d->rows_per_batch % 64 != 0 || d->rows % d->rows_per_batch != 0)
    return dit_fail(ICSA_ERR_INVALID, "norm_rope_pool: rows_per_batch=%d must be a multiple of 64 dividing rows=%d",
                    d->rows_per_batch, d->rows);
  if (pd->mean_batch_stride % 4 || pd->mean_group_stride % 4 || pd->mean_batch_stride < 0 ||
      pd->mean_group_stride < 0)
    return dit_fail(ICSA_ERR_INVALID, "norm_rope_pool: mean strides must be non-negative multiples of 4");
  RopePoolArgs pa{};
  pa.n = a;
  pa.nbl = d->rows_per_batch / 64;
  pa.mb = pd->mean_batch_stride;
  pa.mg = pd->mean_group_stride;
  pa.round_mean = pd->round_mean_bf16 ? 1 : 0;
  RowRmsArgs ra{};
  ra.rows = d->rows; ra.C = d->C; ra.ld = d->ld; ra.eps = d->eps;
  bool any_norm = false;
  for (int j = 0; j < d->count; ++j) {
    if (d->dst_dtype[j] != ICSA_BF16)
      return dit_fail(ICSA_ERR_INVALID, "norm_rope_pool: vector %d must be written as bf16", j);
    if (pd->mean[j] != nullptr && !aligned16(pd->mean[j]))
      return dit_fail(ICSA_ERR_INVALID, "norm_rope_pool: mean %d must be 16-byte aligned", j);
    if (pd->sum[j] != nullptr && !aligned16(pd->sum[j]))
      return dit_fail(ICSA_ERR_INVALID, "norm_rope_pool: sum %d must be 16-byte aligned", j);
    pa.mean[j] = reinterpret_cast<float*>(pd->mean[j]);
    pa.sum[j] = reinterpret_cast<__nv_bfloat16*>(pd->sum[j]);
    pa.bf16_mean[j] = pd->bf16_mean[j] ? 1 : 0;
    ra.src[j] = a.src[j];
    if (d->norm_weight[j] != nullptr) {
      if (pd->rs_scratch == nullptr) return dit_fail(ICSA_ERR_INVALID, "norm_rope_pool: rs_scratch is NULL");
      ra.rs[j] = pd->rs_scratch + size_t(j) * d->rows;
      pa.rs[j] = ra.rs[j];
      any_norm = true;
    }
  }
  if (d->rows == 0) return ICSA_OK;
  if (any_norm) {
    dispatch_chunks(d->C, [&](auto kc) {
      constexpr int KC = decltype(kc)::value;
      row_rms_kernel<KC><<<dim3(d->rows, d->count), kRowThreads, 0, stream>>>(ra);
      return cudaSuccess;
    });
    if ((rc = dit_launch_status("row_rms launch")) != ICSA_OK) return rc;
  }
  const int B = d->rows / d->rows_per_batch;
  const dim3 grid(B * pa.nbl, (d->C + kPoolSlab - 1) / kPoolSlab, d->count);
  norm_rope_pool_kernel<<<grid, kPoolThreadsDit, 0, stream>>>(pa);
  return dit_launch_status("norm_rope_pool launch");
}

int icsa_dit_gated_residual(float* x, const void* y, int64_t ldy, int rows, int C, int rows_per_batch,
                            const float* gate, int64_t gate_batch_stride, cudaStream_t stream) {
  if (x == nullptr || y == nullptr) return dit_fail(ICSA_ERR_INVALID, "gated_residual: NULL buffer");
  if (rows < 0 || C < 8 || C % 8 || ldy < C || ldy % 8 || rows_per_batch < 1)
    return dit_fail(ICSA_ERR_INVALID, "gated_residual: rows=%d C=%d ldy=%lld rows_per_batch=%d", rows, C,
                    (long long)ldy, rows_per_batch);
  if (!aligned16(x) || !aligned16(y) || (gate && (!aligned16(gate) || gate_batch_stride % 4 || gate_batch_stride < 0)))
    return dit_fail(ICSA_ERR_INVALID, "gated_residual: buffers must be 16-byte aligned");
  if (rows == 0) return ICSA_OK;
  GateArgs a{x, reinterpret_cast<const __nv_bfloat16*>(y), ldy, rows, C, rows_per_batch, gate, gate_batch_stride};
  const int64_t n8 = int64_t(rows) * (C / 8);
  const int blocks = int(std::min<int64_t>((n8 + 255) / 256, 148 * 16));
  gated_residual_kernel<<<blocks, 256, 0, stream>>>(a);
  return dit_launch_status("gated_residual launch");
}

}  // extern "C"
