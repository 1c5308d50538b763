// S2: the Gated DeltaNet input side and the gated delta rule, each row resuming from its state in the prefix pool.
//
// Pool geometry (prefix_pool.py of the reference): page p starts at pool + p * page_bytes; a head's recurrent state
// is a (128 key, 128 value) fp32 block at slot (flat head % heads_per_page) of page tables[r][flat / heads_per_page];
// a layer's convolution tail is (3, 6144) bf16 at slot conv_slot of page tables[r][conv_entry].

namespace jb {
namespace gdn {

constexpr int QKV = 6144, ZD = 2048, NH = 16, HDIM = 128;
constexpr int OFF_B = QKV + ZD, OFF_A = QKV + ZD + NH;
constexpr size_t STATE_BYTES = (size_t)HDIM * HDIM * 4;
constexpr size_t CONV_BYTES = (size_t)3 * QKV * 2;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sliding window over tokens: grid (ceil(chunks / 4), 49, rows), 4 warps per block, warp = a chunk of PT tokens of
// one row. Slices 0-47: the 128 channels of one q, k or v head (slice / 16 = part, slice % 16 = head), lane = 4
// channels; the lane keeps its 4 x 4 conv taps and its last three inputs in registers, so every input is read once.
// Slice 48: the gates g and beta of the chunk's tokens (lanes = 2 tokens x 16 heads).
constexpr int PT = 32;

__device__ __forceinline__ void load4(const __nv_bfloat16* src, float (&x)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(src);
  x[0] = bf_lo(u.x);
  x[1] = bf_hi(u.x);
  x[2] = bf_lo(u.y);
  x[3] = bf_hi(u.y);
}

__global__ void __launch_bounds__(128) prep_kernel(const __nv_bfloat16* __restrict__ pr, int ldpr, int n,
                                                   uint8_t* __restrict__ pool, int64_t page_bytes,
                                                   const int* __restrict__ tables, int table_stride, int conv_entry,
                                                   int conv_slot, const float* __restrict__ conv_w,
                                                   const float* __restrict__ a_neg, const float* __restrict__ dt_bias,
                                                   __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                                                   __nv_bfloat16* __restrict__ v, float* __restrict__ g,
                                                   __nv_bfloat16* __restrict__ beta, const int* __restrict__ real,
                                                   const int* __restrict__ out_tables, int out_table_stride) {
  pdl_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.z, slice = blockIdx.y;
  const int t0 = (blockIdx.x * 4 + warp) * PT;
  if (t0 >= n) return;
  const int t1 = min(t0 + PT, n);
  const size_t rbase = (size_t)row * n;
  if (slice == 3 * NH) {
    const int h = lane & 15;
    const float an = a_neg[h], db = dt_bias[h];
    const int rl = real ? real[row] : n;
    for (int tt = t0 + (lane >> 4); tt < t1; tt += 2) {
      const size_t t = rbase + tt;
      const float bv = __bfloat162float(pr[t * ldpr + OFF_B + h]);
      const float av = __bfloat162float(pr[t * ldpr + OFF_A + h]) + db;
      const float sp = av > 20.0f ? av : logf(1.0f + expf(av));
      float gv = an * sp;
      float bt = 1.0f / (1.0f + expf(-bv));
      if (tt >= rl) {
        gv = 0.f;
        bt = 0.f;
      }
      g[t * NH + h] = gv;
      beta[t * NH + h] = __float2bfloat16_rn(bt);
    }
    return;
  }
  const int part = slice / NH, head = slice % NH;
  const int ch = part * 2048 + head * HDIM + lane * 4;
  const int page = tables[(size_t)row * table_stride + conv_entry];
  const __nv_bfloat16* tail = reinterpret_cast<const __nv_bfloat16*>(pool + (int64_t)page * page_bytes +
                                                                      conv_slot * CONV_BYTES);
  float w[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 wv = *reinterpret_cast<const float4*>(conv_w + (size_t)i * QKV + ch);
    w[i][0] = wv.x;
    w[i][1] = wv.y;
    w[i][2] = wv.z;
    w[i][3] = wv.w;
  }
  // inputs at positions t0 - 3 .. t0 - 1 of [3 cached; new]
  float x0[4], x1[4], x2[4];
  {
    const int p0 = t0 - 3, p1 = t0 - 2, p2 = t0 - 1;
    load4(p0 < 0 ? tail + (size_t)(p0 + 3) * QKV + ch : pr + (rbase + p0) * ldpr + ch, x0);
    load4(p1 < 0 ? tail + (size_t)(p1 + 3) * QKV + ch : pr + (rbase + p1) * ldpr + ch, x1);
    load4(p2 < 0 ? tail + (size_t)(p2 + 3) * QKV + ch : pr + (rbase + p2) * ldpr + ch, x2);
  }
  __nv_bfloat16* dst = part == 0 ? q : (part == 1 ? k : v);
  // tokens in groups of 8: the group's 8 loads are issued before any of them is used
  for (int tb = t0; tb < t1; tb += 8) {
    uint2 raw[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      raw[u] = *reinterpret_cast<const uint2*>(pr + (rbase + min(tb + u, t1 - 1)) * ldpr + ch);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int tt = tb + u;
      if (tt >= t1) break;   // the same for the whole warp
      const float x3[4] = {bf_lo(raw[u].x), bf_hi(raw[u].x), bf_lo(raw[u].y), bf_hi(raw[u].y)};
      float c[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float acc = 0.f;
        acc += w[0][e] * x0[e];
        acc += w[1][e] * x1[e];
        acc += w[2][e] * x2[e];
        acc += w[3][e] * x3[e];
        // SiLU with the fast intrinsics (the result is rounded to bf16 at once; __fdividef(x, inf) = 0 is the limit)
        c[e] = round_bf(__fdividef(acc, 1.0f + __expf(-acc)));
        x0[e] = x1[e];
        x1[e] = x2[e];
        x2[e] = x3[e];
      }
      const size_t o = ((rbase + tt) * NH + head) * HDIM + lane * 4;
      if (part < 2) {
        const float ss = warp_sum(c[0] * c[0] + c[1] * c[1] + c[2] * c[2] + c[3] * c[3]);
        const float rs = rsqrtf(ss + 1e-6f);
        *reinterpret_cast<uint2*>(dst + o) =
            make_uint2(pack_bf2(c[0] * rs, c[1] * rs), pack_bf2(c[2] * rs, c[3] * rs));
      } else {
        *reinterpret_cast<uint2*>(dst + o) = make_uint2(pack_bf2(c[0], c[1]), pack_bf2(c[2], c[3]));
      }
    }
  }
  if (real && out_tables && t0 == 0) {
    // the prefix pass: this row's last three real convolution inputs become its cached tail
    const int r = real[row];
    const int opage = out_tables[(size_t)row * out_table_stride + conv_entry];
    __nv_bfloat16* otail = reinterpret_cast<__nv_bfloat16*>(pool + (int64_t)opage * page_bytes + conv_slot * CONV_BYTES);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const int pos = r - 3 + i;
      uint2 val;
      if (pos < 0) val = *reinterpret_cast<const uint2*>(tail + (size_t)(pos + 3) * QKV + ch);
      else val = *reinterpret_cast<const uint2*>(pr + (rbase + pos) * ldpr + ch);
      *reinterpret_cast<uint2*>(otail + (size_t)i * QKV + ch) = val;
    }
  }
}

// One CTA per (row, head), 256 threads: the thread pair (2j, 2j + 1) holds value column j of the (128 x 128) fp32
// state, key rows [0, 64) and [64, 128), in registers; pair sums by one shuffle. Per token:
// a = S^T k (old state), v' = beta (v - e^g a), S = e^g S + k v'^T, o = S^T q / sqrt(128).
__global__ void __launch_bounds__(256) scan_kernel(const __nv_bfloat16* __restrict__ q,
                                                   const __nv_bfloat16* __restrict__ k,
                                                   const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
                                                   const __nv_bfloat16* __restrict__ beta,
                                                   __nv_bfloat16* __restrict__ o, int n, uint8_t* __restrict__ pool,
                                                   int64_t page_bytes, const int* __restrict__ tables,
                                                   int table_stride, int first_head, int heads_per_page,
                                                   const int* __restrict__ last, const int* __restrict__ out_tables,
                                                   int out_table_stride) {
  pdl_begin();
  constexpr int HALF = HDIM / 2;
  __shared__ __align__(16) float kq[2][2][HDIM];
  const int row = blockIdx.x / NH, h = blockIdx.x % NH;
  const int j = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int i0 = half * HALF;
  const int flat = first_head + h;
  const int page = tables[(size_t)row * table_stride + flat / heads_per_page];
  const float* s_in = reinterpret_cast<const float*>(pool + (int64_t)page * page_bytes +
                                                     (flat % heads_per_page) * STATE_BYTES);
  float S[HALF];
#pragma unroll
  for (int i = 0; i < HALF; ++i) S[i] = s_in[(i0 + i) * HDIM + j];
  const int stop = last ? min(last[row] + 1, n) : n;
  const float scale = rsqrtf((float)HDIM);
  for (int tt = 0; tt < stop; ++tt) {
    const size_t tok = (size_t)row * n + tt;
    const size_t base = (tok * NH + h) * HDIM;
    const int buf = tt & 1;
    if (threadIdx.x < HDIM) {
      kq[buf][0][threadIdx.x] = __bfloat162float(k[base + threadIdx.x]);
      kq[buf][1][threadIdx.x] = __bfloat162float(q[base + threadIdx.x]) * scale;
    }
    const float vj = __bfloat162float(v[base + j]);
    const float gt = g[tok * NH + h];
    const float bt = __bfloat162float(beta[tok * NH + h]);
    __syncthreads();
    const float4* k4 = reinterpret_cast<const float4*>(kq[buf][0] + i0);
    const float4* q4 = reinterpret_cast<const float4*>(kq[buf][1] + i0);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < HALF / 4; ++i) {
      const float4 kk = k4[i];
      a0 = fmaf(S[4 * i + 0], kk.x, a0);
      a1 = fmaf(S[4 * i + 1], kk.y, a1);
      a0 = fmaf(S[4 * i + 2], kk.z, a0);
      a1 = fmaf(S[4 * i + 3], kk.w, a1);
    }
    float a = a0 + a1;
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    const float eg = expf(gt);
    const float vnew = bt * (vj - eg * a);
    float o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int i = 0; i < HALF / 4; ++i) {
      const float4 kk = k4[i];
      const float4 qq = q4[i];
      S[4 * i + 0] = fmaf(S[4 * i + 0], eg, kk.x * vnew);
      S[4 * i + 1] = fmaf(S[4 * i + 1], eg, kk.y * vnew);
      S[4 * i + 2] = fmaf(S[4 * i + 2], eg, kk.z * vnew);
      S[4 * i + 3] = fmaf(S[4 * i + 3], eg, kk.w * vnew);
      o0 = fmaf(S[4 * i + 0], qq.x, o0);
      o1 = fmaf(S[4 * i + 1], qq.y, o1);
      o0 = fmaf(S[4 * i + 2], qq.z, o0);
      o1 = fmaf(S[4 * i + 3], qq.w, o1);
    }
    float ov = o0 + o1;
    ov += __shfl_xor_sync(0xffffffffu, ov, 1);
    if (half == 0) o[base + j] = __float2bfloat16_rn(ov);
  }
  if (half == 0)
    for (int tt = stop; tt < n; ++tt) o[(((size_t)row * n + tt) * NH + h) * HDIM + j] = __float2bfloat16_rn(0.f);
  if (out_tables) {
    const int opage = out_tables[(size_t)row * out_table_stride + flat / heads_per_page];
    float* s_out = reinterpret_cast<float*>(pool + (int64_t)opage * page_bytes + (flat % heads_per_page) * STATE_BYTES);
#pragma unroll
    for (int i = 0; i < HALF; ++i) s_out[(i0 + i) * HDIM + j] = S[i];
  }
}

}  // namespace gdn
}  // namespace jb

using namespace jb;

extern "C" int jb_gdn_prep_rows(const uint16_t* pr, int ldpr, int t, int n, void* pool, int64_t page_bytes,
                                const int32_t* tables, int table_stride, int conv_entry, int conv_slot,
                                const float* conv_w, const float* a_neg, const float* dt_bias, uint16_t* q,
                                uint16_t* k, uint16_t* v, float* g, uint16_t* beta, const int32_t* real,
                                const int32_t* out_tables, int out_table_stride, void* stream) {
  JB_REQUIRE(pr && pool && tables && conv_w && a_neg && dt_bias && q && k && v && g && beta,
             "jb_gdn_prep_rows: null pointer");
  JB_REQUIRE(t > 0 && n > 0 && t % n == 0, "jb_gdn_prep_rows: a pass of %d tokens in rows of %d", t, n);
  JB_REQUIRE(ldpr >= gdn::OFF_A + gdn::NH && ldpr % 4 == 0, "jb_gdn_prep_rows: ldpr %d", ldpr);
  JB_REQUIRE(conv_entry >= 0 && conv_entry < table_stride && conv_slot >= 0 &&
                 (int64_t)(conv_slot + 1) * (int64_t)gdn::CONV_BYTES <= page_bytes,
             "jb_gdn_prep_rows: conv entry %d / slot %d do not fit the page geometry", conv_entry, conv_slot);
  JB_REQUIRE(!out_tables || real, "jb_gdn_prep_rows: out_tables needs real");
  const int chunks = (n + gdn::PT - 1) / gdn::PT;
  dim3 grid((chunks + 3) / 4, 3 * gdn::NH + 1, t / n);
  launch_pdl(gdn::prep_kernel, grid, 128, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(pr), ldpr, n, static_cast<uint8_t*>(pool), page_bytes, tables,
      table_stride, conv_entry, conv_slot, conv_w, a_neg, dt_bias, reinterpret_cast<__nv_bfloat16*>(q),
      reinterpret_cast<__nv_bfloat16*>(k), reinterpret_cast<__nv_bfloat16*>(v), g,
      reinterpret_cast<__nv_bfloat16*>(beta), real, out_tables, out_table_stride);
  return check_launch("gdn prep_kernel");
}

extern "C" int jb_gdn_scan_recurrent(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                           const uint16_t* beta, uint16_t* o, int b, int n, void* pool, int64_t page_bytes,
                           const int32_t* tables, int table_stride, int first_head, int heads_per_page,
                           const int32_t* last, const int32_t* out_tables, int out_table_stride, void* stream) {
  JB_REQUIRE(q && k && v && g && beta && o && pool && tables, "jb_gdn_scan_recurrent: null pointer");
  JB_REQUIRE(b > 0 && n > 0, "jb_gdn_scan_recurrent: b %d, n %d", b, n);
  JB_REQUIRE(heads_per_page > 0 && (int64_t)heads_per_page * (int64_t)gdn::STATE_BYTES <= page_bytes,
             "jb_gdn_scan_recurrent: %d heads per page do not fit pages of %lld bytes", heads_per_page,
             (long long)page_bytes);
  JB_REQUIRE(first_head >= 0 && (first_head + gdn::NH - 1) / heads_per_page < table_stride,
             "jb_gdn_scan_recurrent: heads %d.. reach past the block table (%d entries)", first_head, table_stride);
  launch_pdl(gdn::scan_kernel, b * gdn::NH, 256, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      reinterpret_cast<const __nv_bfloat16*>(v), g, reinterpret_cast<const __nv_bfloat16*>(beta),
      reinterpret_cast<__nv_bfloat16*>(o), n, static_cast<uint8_t*>(pool), page_bytes, tables, table_stride,
      first_head, heads_per_page, last, out_tables, out_table_stride);
  return check_launch("gdn scan_kernel");
}
