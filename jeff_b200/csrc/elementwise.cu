// S4 (first form): the fused norms and activations between the products, and the per-row readout. Each keeps the
// reference's bf16 rounding points (fast_path.py:75-156, batched_kernels.py:492-552); HBM-bound elementwise work with
// 16-byte vector accesses.

namespace jb {
namespace ew {

constexpr float EPS = 1e-6f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// block-wide sum for blockDim <= 1024 (scratch: 32 floats)
__device__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < nw ? scratch[lane] : 0.f;
  return warp_sum(t);
}
__device__ float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < nw ? scratch[lane] : -INFINITY;
  return warp_max(t);
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  f[0] = bf_lo(u.x); f[1] = bf_hi(u.x); f[2] = bf_lo(u.y); f[3] = bf_hi(u.y);
  f[4] = bf_lo(u.z); f[5] = bf_hi(u.z); f[6] = bf_lo(u.w); f[7] = bf_hi(u.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf2(f[0], f[1]), pack_bf2(f[2], f[3]), pack_bf2(f[4], f[5]), pack_bf2(f[6], f[7]));
}

constexpr int RMS_MAX_VEC = 4;   // n <= 128 threads * 4 vectors * 8 = 4096

// xo = bf16(x + d); h = bf16(xo * rsqrt(mean(xo^2) + eps) * w1)
__global__ void __launch_bounds__(128) add_rms_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ d,
                                                      const float* __restrict__ w1, __nv_bfloat16* xo,
                                                      __nv_bfloat16* __restrict__ h, int n) {
  pdl_begin();
  __shared__ float scratch[32];
  const size_t row = blockIdx.x;
  const int nvec = n / 8;
  float v[RMS_MAX_VEC][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < RMS_MAX_VEC; ++j) {
    const int c = threadIdx.x + j * 128;
    if (c < nvec) {
      uint4 xu = reinterpret_cast<const uint4*>(x + row * n)[c];
      unpack8(xu, v[j]);
      if (d) {
        float dv[8];
        unpack8(reinterpret_cast<const uint4*>(d + row * n)[c], dv);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[j][e] = round_bf(v[j][e] + dv[e]);
        reinterpret_cast<uint4*>(xo + row * n)[c] = pack8(v[j]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[j][e] * v[j][e];
    }
  }
  const float rs = rsqrtf(block_sum(ss, scratch) / n + EPS);
#pragma unroll
  for (int j = 0; j < RMS_MAX_VEC; ++j) {
    const int c = threadIdx.x + j * 128;
    if (c < nvec) {
      float o[8];
      const float4 wa = reinterpret_cast<const float4*>(w1)[2 * c];
      const float4 wb = reinterpret_cast<const float4*>(w1)[2 * c + 1];
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[j][e] * rs * w[e];
      reinterpret_cast<uint4*>(h + row * n)[c] = pack8(o);
    }
  }
}

// the same for rows of 1024: one warp per row (4 x 16 bytes per lane), 4 rows per block, no block barriers
__global__ void __launch_bounds__(128) add_rms_1024_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ d,
                                                           const float* __restrict__ w1, __nv_bfloat16* xo,
                                                           __nv_bfloat16* __restrict__ h, int rows) {
  pdl_begin();
  constexpr int N = 1024;
  const int lane = threadIdx.x & 31;
  const size_t row = (size_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= (size_t)rows) return;
  float v[4][8];
  uint4 xu[4], du[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) xu[j] = reinterpret_cast<const uint4*>(x + row * N)[lane + 32 * j];
  if (d) {
#pragma unroll
    for (int j = 0; j < 4; ++j) du[j] = reinterpret_cast<const uint4*>(d + row * N)[lane + 32 * j];
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    unpack8(xu[j], v[j]);
    if (d) {
      float dv[8];
      unpack8(du[j], dv);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = round_bf(v[j][e] + dv[e]);
      reinterpret_cast<uint4*>(xo + row * N)[lane + 32 * j] = pack8(v[j]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[j][e] * v[j][e];
  }
  const float rs = rsqrtf(warp_sum(ss) / N + EPS);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane + 32 * j;
    const float4 wa = reinterpret_cast<const float4*>(w1)[2 * c];
    const float4 wb = reinterpret_cast<const float4*>(w1)[2 * c + 1];
    const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = v[j][e] * rs * w[e];
    reinterpret_cast<uint4*>(h + row * N)[c] = pack8(o);
  }
}

// hidden[b] = bf16(rms(bf16(x[t] + d[t])) * w1), t = b * row_len + last[b]
__global__ void __launch_bounds__(128) rms_last_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ d,
                                                       const int* __restrict__ last, int row_len, int n,
                                                       const float* __restrict__ w1,
                                                       __nv_bfloat16* __restrict__ hidden) {
  pdl_begin();
  __shared__ float scratch[32];
  const size_t t = (size_t)blockIdx.x * row_len + last[blockIdx.x];
  const int nvec = n / 8;
  float v[RMS_MAX_VEC][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < RMS_MAX_VEC; ++j) {
    const int c = threadIdx.x + j * 128;
    if (c < nvec) {
      float dv[8];
      unpack8(reinterpret_cast<const uint4*>(x + t * n)[c], v[j]);
      unpack8(reinterpret_cast<const uint4*>(d + t * n)[c], dv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[j][e] = round_bf(v[j][e] + dv[e]);
        ss += v[j][e] * v[j][e];
      }
    }
  }
  const float rs = rsqrtf(block_sum(ss, scratch) / n + EPS);
#pragma unroll
  for (int j = 0; j < RMS_MAX_VEC; ++j) {
    const int c = threadIdx.x + j * 128;
    if (c < nvec) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[j][e] * rs * w1[8 * c + e];
      reinterpret_cast<uint4*>(hidden + (size_t)blockIdx.x * n)[c] = pack8(o);
    }
  }
}

__global__ void embed_kernel(const __nv_bfloat16* __restrict__ table, int vocab, int dim,
                             const int* __restrict__ ids, int t, __nv_bfloat16* __restrict__ x) {
  pdl_begin();
  const int nvec = dim / 8;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)t * nvec) return;
  const size_t tok = i / nvec;
  const int c = (int)(i % nvec);
  int id = ids[tok];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  reinterpret_cast<uint4*>(x + tok * dim)[c] = reinterpret_cast<const uint4*>(table + (size_t)id * dim)[c];
}

__device__ __forceinline__ float silu_rounded(float g) { return round_bf(g / (1.0f + expf(-g))); }
__device__ __forceinline__ float sigmoid(float g) { return 1.0f / (1.0f + expf(-g)); }

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int ldgu, int inter,
                                __nv_bfloat16* __restrict__ y, int rows) {
  pdl_begin();
  const int nvec = inter / 8;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * nvec) return;
  const size_t r = i / nvec;
  const int c = (int)(i % nvec);
  float g[8], u[8], o[8];
  unpack8(reinterpret_cast<const uint4*>(gu + r * ldgu)[c], g);
  unpack8(reinterpret_cast<const uint4*>(gu + r * ldgu + inter)[c], u);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = silu_rounded(g[e]) * u[e];
  reinterpret_cast<uint4*>(y + r * inter)[c] = pack8(o);
}

// o (rows, 8, 256); gate of head h at pr[r, h * 512 + 256 + d]
__global__ void gate_mul_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ pr, int ldpr,
                                __nv_bfloat16* __restrict__ y, int rows) {
  pdl_begin();
  constexpr int NVEC = 8 * 256 / 8;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * NVEC) return;
  const size_t r = i / NVEC;
  const int c = (int)(i % NVEC);
  const int h = c / 32, dv = c % 32;
  float ov[8], gv[8], out[8];
  unpack8(reinterpret_cast<const uint4*>(o + r * 2048)[c], ov);
  unpack8(reinterpret_cast<const uint4*>(pr + r * ldpr + h * 512 + 256)[dv], gv);
#pragma unroll
  for (int e = 0; e < 8; ++e) out[e] = ov[e] * round_bf(sigmoid(gv[e]));
  reinterpret_cast<uint4*>(y + r * 2048)[c] = pack8(out);
}

// one half-warp per (token, head of 128), 8 channels per lane: y = bf16(bf16(w * bf16(rms(o))) * silu(z))
__global__ void gated_norm_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ pr, int ldpr,
                                  int z_off, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                  int rows) {
  pdl_begin();
  const size_t pair = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;   // (token, head) index
  const int sub = threadIdx.x & 15;
  const bool live = pair < (size_t)rows * 16;
  const size_t r = live ? pair / 16 : 0;
  const int h = live ? (int)(pair % 16) : 0;
  float v[8], z[8], wv[8];
  unpack8(reinterpret_cast<const uint4*>(o + (r * 16 + h) * 128)[sub], v);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rs = rsqrtf(ss / 128.f + EPS);
  unpack8(reinterpret_cast<const uint4*>(pr + r * ldpr + z_off + h * 128)[sub], z);
  unpack8(reinterpret_cast<const uint4*>(w)[sub], wv);
  float out[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float nv = round_bf(v[e] * rs);
    const float gw = round_bf(wv[e] * nv);
    out[e] = gw * (z[e] / (1.0f + expf(-z[e])));
  }
  if (live)
    reinterpret_cast<uint4*>(y + r * 2048 + h * 128)[sub] =
        make_uint4(pack_bf2(out[0], out[1]), pack_bf2(out[2], out[3]), pack_bf2(out[4], out[5]),
                   pack_bf2(out[6], out[7]));
}

// one block of 256 threads per row: 255 logits = bf16(W[a] . h) (fp32 sums), mask, temperature, softmax
__global__ void __launch_bounds__(256) readout_kernel(const __nv_bfloat16* __restrict__ hidden,
                                                      const __nv_bfloat16* __restrict__ pool, int pool_rows,
                                                      const float* __restrict__ temp_pool,
                                                      const int* __restrict__ adapters, const int* __restrict__ counts,
                                                      float* __restrict__ probs) {
  pdl_begin();
  __shared__ float logits[256];
  __shared__ float scratch[32];
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int a = adapters[b];
  if (a < 0 || a >= pool_rows) a = 0;
  float hv[4][8];
#pragma unroll
  for (int j = 0; j < 4; ++j) unpack8(reinterpret_cast<const uint4*>(hidden + (size_t)b * 1024)[lane + 32 * j], hv[j]);
  const __nv_bfloat16* W = pool + (size_t)a * 255 * 1024;
  for (int o = warp; o < 255; o += 8) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float wv[8];
      unpack8(reinterpret_cast<const uint4*>(W + (size_t)o * 1024)[lane + 32 * j], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += wv[e] * hv[j][e];
    }
    acc = warp_sum(acc);
    if (lane == 0) logits[o] = round_bf(acc);
  }
  __syncthreads();
  const int count = counts[b];
  const float temp = temp_pool[a];
  const int o = threadIdx.x;
  float x = -INFINITY;
  if (o < 255) x = ((o < count) ? logits[o] : -1e9f) / temp;
  const float mx = block_max(x, scratch);
  const float e = (o < 255) ? expf(x - mx) : 0.f;
  const float sum = block_sum(e, scratch);
  if (o < 255) probs[(size_t)b * 255 + o] = e / sum;
}

}  // namespace ew
}  // namespace jb

using namespace jb;

static inline unsigned blocks_for(size_t n, unsigned threads) { return (unsigned)((n + threads - 1) / threads); }

extern "C" int jb_add_rms(const uint16_t* x, const uint16_t* d, const float* w1, uint16_t* xo, uint16_t* h, int rows,
                          int n, void* stream) {
  JB_REQUIRE(x && w1 && h, "jb_add_rms: null pointer");
  JB_REQUIRE(!d || xo, "jb_add_rms: xo is needed with d");
  JB_REQUIRE(rows > 0 && n > 0 && n % 8 == 0 && n <= 128 * ew::RMS_MAX_VEC * 8, "jb_add_rms: rows %d, n %d", rows, n);
  if (n == 1024) {
    launch_pdl(ew::add_rms_1024_kernel, (rows + 3) / 4, 128, 0, (cudaStream_t)stream,
        reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(d), w1,
        reinterpret_cast<__nv_bfloat16*>(xo), reinterpret_cast<__nv_bfloat16*>(h), rows);
    return check_launch("add_rms_1024_kernel");
  }
  launch_pdl(ew::add_rms_kernel, rows, 128, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(d), w1,
      reinterpret_cast<__nv_bfloat16*>(xo), reinterpret_cast<__nv_bfloat16*>(h), n);
  return check_launch("add_rms_kernel");
}

extern "C" int jb_rms_last(const uint16_t* x, const uint16_t* d, const int32_t* last, int b, int row_len, int n,
                           const float* w1, uint16_t* hidden, void* stream) {
  JB_REQUIRE(x && d && last && w1 && hidden, "jb_rms_last: null pointer");
  JB_REQUIRE(b > 0 && row_len > 0 && n > 0 && n % 8 == 0 && n <= 128 * ew::RMS_MAX_VEC * 8,
             "jb_rms_last: b %d, row_len %d, n %d", b, row_len, n);
  launch_pdl(ew::rms_last_kernel, b, 128, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(d), last, row_len, n, w1,
      reinterpret_cast<__nv_bfloat16*>(hidden));
  return check_launch("rms_last_kernel");
}

extern "C" int jb_embed(const uint16_t* table, int vocab, int dim, const int32_t* ids, int t, uint16_t* x,
                        void* stream) {
  JB_REQUIRE(table && ids && x, "jb_embed: null pointer");
  JB_REQUIRE(vocab > 0 && dim > 0 && dim % 8 == 0 && t > 0, "jb_embed: vocab %d, dim %d, t %d", vocab, dim, t);
  const size_t n = (size_t)t * (dim / 8);
  launch_pdl(ew::embed_kernel, blocks_for(n, 256), 256, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(table), vocab, dim, ids, t, reinterpret_cast<__nv_bfloat16*>(x));
  return check_launch("embed_kernel");
}

extern "C" int jb_silu_mul(const uint16_t* gu, int ldgu, int inter, uint16_t* y, int rows, void* stream) {
  JB_REQUIRE(gu && y, "jb_silu_mul: null pointer");
  JB_REQUIRE(rows > 0 && inter > 0 && inter % 8 == 0 && ldgu >= 2 * inter && ldgu % 8 == 0,
             "jb_silu_mul: rows %d, inter %d, ldgu %d", rows, inter, ldgu);
  const size_t n = (size_t)rows * (inter / 8);
  launch_pdl(ew::silu_mul_kernel, blocks_for(n, 256), 256, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(gu), ldgu, inter, reinterpret_cast<__nv_bfloat16*>(y), rows);
  return check_launch("silu_mul_kernel");
}

extern "C" int jb_gate_mul(const uint16_t* o, const uint16_t* pr, int ldpr, uint16_t* y, int rows, void* stream) {
  JB_REQUIRE(o && pr && y, "jb_gate_mul: null pointer");
  JB_REQUIRE(rows > 0 && ldpr >= 4096 && ldpr % 8 == 0, "jb_gate_mul: rows %d, ldpr %d", rows, ldpr);
  const size_t n = (size_t)rows * 256;
  launch_pdl(ew::gate_mul_kernel, blocks_for(n, 256), 256, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(o), reinterpret_cast<const __nv_bfloat16*>(pr), ldpr,
      reinterpret_cast<__nv_bfloat16*>(y), rows);
  return check_launch("gate_mul_kernel");
}

extern "C" int jb_gated_norm(const uint16_t* o, const uint16_t* pr, int ldpr, int z_off, const uint16_t* w,
                             uint16_t* y, int rows, void* stream) {
  JB_REQUIRE(o && pr && w && y, "jb_gated_norm: null pointer");
  JB_REQUIRE(rows > 0 && z_off >= 0 && z_off % 8 == 0 && ldpr >= z_off + 2048 && ldpr % 8 == 0,
             "jb_gated_norm: rows %d, ldpr %d, z_off %d (multiples of 8)", rows, ldpr, z_off);
  JB_REQUIRE(((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(pr) | reinterpret_cast<uintptr_t>(w) |
               reinterpret_cast<uintptr_t>(y)) & 15) == 0,
             "jb_gated_norm: o, pr, w and y must be 16-byte aligned");
  const size_t threads = (size_t)rows * 16 * 16;   // 16 per (token, head)
  launch_pdl(ew::gated_norm_kernel, blocks_for(threads, 256), 256, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(o), reinterpret_cast<const __nv_bfloat16*>(pr), ldpr, z_off,
      reinterpret_cast<const __nv_bfloat16*>(w), reinterpret_cast<__nv_bfloat16*>(y), rows);
  return check_launch("gated_norm_kernel");
}

extern "C" int jb_readout_rows(const uint16_t* hidden, const uint16_t* readout_pool, int pool_rows,
                               const float* temp_pool, const int32_t* adapters, const int32_t* counts, int b,
                               float* probs, void* stream) {
  JB_REQUIRE(hidden && readout_pool && temp_pool && adapters && counts && probs, "jb_readout_rows: null pointer");
  JB_REQUIRE(b > 0 && pool_rows > 0, "jb_readout_rows: b %d, pool_rows %d", b, pool_rows);
  launch_pdl(ew::readout_kernel, b, 256, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(hidden), reinterpret_cast<const __nv_bfloat16*>(readout_pool),
      pool_rows, temp_pool, adapters, counts, probs);
  return check_launch("readout_kernel");
}
