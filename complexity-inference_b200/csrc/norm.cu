// Row-wise kernels on the f32 residual stream: embedding lookup, fused
// partial-sum reduction + residual add + RMSNorm (+ mu_clamp at each of the
// reference's clamp sites), final-norm row gather, and the INL dynamics step
// of DeepForCausalLM with its post-attention norm and mu-guided routing.
//
// One CTA per token row; the row is staged in shared memory (hidden <= 16384)
// so the norm needs a single HBM read of every input.  These kernels are
// HBM-bound: per row they move (num_partials + 2)·4·H bytes in and 6·H out.
#include <math.h>

#include "abi_util.h"
#include "common.cuh"

namespace muk {

constexpr int kRowThreads = 256;
constexpr int kMaxHidden = 16384;

struct ClampArgs {
  float mu, cmin, cmax;
};

// ---------------------------------------------------------------------------
__global__ void embed_kernel(const int32_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             int64_t table_stride, float* __restrict__ resid, int hidden, int vocab,
                             ClampParams cp) {
  const int t = blockIdx.x;
  const int id = ids[t];
  float* out = resid + (int64_t)t * hidden;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_device_error(kDevBadIndex);
    for (int j = threadIdx.x; j < hidden; j += blockDim.x) out[j] = 0.f;
    return;
  }
  const __nv_bfloat16* row = table + (int64_t)id * table_stride;
  for (int j = threadIdx.x * 2; j < hidden; j += blockDim.x * 2) {
    float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(row + j));
    out[j] = mu_clamp(v.x, cp);
    out[j + 1] = mu_clamp(v.y, cp);
  }
}

// Four consecutive delta values as a float4, from f32 or bf16 rows (index in
// units of 4 elements).
__device__ __forceinline__ float4 load4(const float* p, int64_t i4) {
  return reinterpret_cast<const float4*>(p)[i4];
}
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p, int64_t i4) {
  const uint2 u = reinterpret_cast<const uint2*>(p)[i4];
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  return make_float4(a.x, a.y, b.x, b.y);
}

// ---------------------------------------------------------------------------
template <typename DT>
__global__ void residual_rmsnorm_kernel(float* __restrict__ resid, const DT* __restrict__ partials,
                                        int64_t partial_stride, int64_t partial_row_stride,
                                        int num_partials, const int32_t* __restrict__ delta_rows,
                                        const float* __restrict__ norm_w, float eps,
                                        __nv_bfloat16* __restrict__ out, int64_t out_stride,
                                        int hidden, int clamp_delta, int clamp_sum,
                                        ClampParams cp_norm, ClampParams cp) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  extern __shared__ float srow[];
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int src = delta_rows ? delta_rows[t] : t;
  float* rrow = resid + (int64_t)t * hidden;
  float ss = 0.f;
  for (int j = threadIdx.x * 4; j < hidden; j += blockDim.x * 4) {
    float4 r = *reinterpret_cast<const float4*>(rrow + j);
    if (num_partials > 0) {
      float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = 0; p < num_partials; ++p) {
        float4 x = load4(partials + p * partial_stride + (int64_t)src * partial_row_stride, j / 4);
        d.x += x.x;
        d.y += x.y;
        d.z += x.z;
        d.w += x.w;
      }
      if (clamp_delta) {
        d.x = mu_clamp(d.x, cp);
        d.y = mu_clamp(d.y, cp);
        d.z = mu_clamp(d.z, cp);
        d.w = mu_clamp(d.w, cp);
      }
      r.x += d.x;
      r.y += d.y;
      r.z += d.z;
      r.w += d.w;
      if (clamp_sum) {
        r.x = mu_clamp(r.x, cp);
        r.y = mu_clamp(r.y, cp);
        r.z = mu_clamp(r.z, cp);
        r.w = mu_clamp(r.w, cp);
      }
      *reinterpret_cast<float4*>(rrow + j) = r;
    }
    *reinterpret_cast<float4*>(srow + j) = r;
    ss += r.x * r.x + r.y * r.y + r.z * r.z + r.w * r.w;
  }
  if (out == nullptr) return;
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total / (float)hidden + eps);
  __nv_bfloat16* orow = out + (int64_t)t * out_stride;
  for (int j = threadIdx.x * 2; j < hidden; j += blockDim.x * 2) {
    float a = mu_clamp(norm_w[j] * (srow[j] * inv), cp_norm);
    float b = mu_clamp(norm_w[j + 1] * (srow[j + 1] * inv), cp_norm);
    *reinterpret_cast<uint32_t*>(orow + j) = pack_bf16x2(a, b);
  }
}

// ---------------------------------------------------------------------------
// Same computation with the row held in registers: blockDim.x * VPT float4
// = hidden, every load of a row issued before the first use (the generic
// kernel above serialises them on its strided loop).
template <int VPT, typename DT>
__global__ void __launch_bounds__(256, VPT <= 4 ? 4 : (VPT <= 8 ? 2 : 1))
    residual_rmsnorm_vec_kernel(float* __restrict__ resid, const DT* __restrict__ partials,
                                int64_t partial_stride, int64_t partial_row_stride,
                                int num_partials, const int32_t* __restrict__ delta_rows,
                                const float* __restrict__ norm_w, float eps,
                                __nv_bfloat16* __restrict__ out, int64_t out_stride, int hidden,
                                int clamp_delta, int clamp_sum, ClampParams cp_norm,
                                ClampParams cp) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int src = delta_rows ? delta_rows[t] : t;
  float4* rrow = reinterpret_cast<float4*>(resid + (int64_t)t * hidden);
  const int n = blockDim.x;
  float4 r[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) r[i] = rrow[threadIdx.x + i * n];
  if (num_partials > 0) {
    float4 d[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) d[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < num_partials; ++p) {
      const DT* prow = partials + p * partial_stride + (int64_t)src * partial_row_stride;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const float4 x = load4(prow, threadIdx.x + i * n);
        d[i].x += x.x;
        d[i].y += x.y;
        d[i].z += x.z;
        d[i].w += x.w;
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (clamp_delta) {
        d[i].x = mu_clamp(d[i].x, cp);
        d[i].y = mu_clamp(d[i].y, cp);
        d[i].z = mu_clamp(d[i].z, cp);
        d[i].w = mu_clamp(d[i].w, cp);
      }
      r[i].x += d[i].x;
      r[i].y += d[i].y;
      r[i].z += d[i].z;
      r[i].w += d[i].w;
      if (clamp_sum) {
        r[i].x = mu_clamp(r[i].x, cp);
        r[i].y = mu_clamp(r[i].y, cp);
        r[i].z = mu_clamp(r[i].z, cp);
        r[i].w = mu_clamp(r[i].w, cp);
      }
      rrow[threadIdx.x + i * n] = r[i];
    }
  }
  if (out == nullptr) return;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) ss += r[i].x * r[i].x + r[i].y * r[i].y + r[i].z * r[i].z + r[i].w * r[i].w;
  const float inv = rsqrtf(block_sum(ss, red) / (float)hidden + eps);
  const float4* w4 = reinterpret_cast<const float4*>(norm_w);
  uint2* orow = reinterpret_cast<uint2*>(out + (int64_t)t * out_stride);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const float4 w = w4[threadIdx.x + i * n];
    uint2 o;
    o.x = pack_bf16x2(mu_clamp(w.x * (r[i].x * inv), cp_norm), mu_clamp(w.y * (r[i].y * inv), cp_norm));
    o.y = pack_bf16x2(mu_clamp(w.z * (r[i].z * inv), cp_norm), mu_clamp(w.w * (r[i].w * inv), cp_norm));
    orow[threadIdx.x + i * n] = o;
  }
}

// float4s per thread for the register-resident row kernels (0: use the
// generic kernel): 256 threads when hidden is a multiple of 1024, else one
// float4 per thread for hidden <= 4096 in whole warps.
static int row_vpt(int hidden) {
  if (hidden % 1024 == 0 && hidden / 1024 <= 16) return hidden / 1024;
  if (hidden % 128 == 0 && hidden <= 4096) return -1;  // VPT 1, hidden / 4 threads
  return 0;
}

__global__ void rmsnorm_rows_kernel(const float* __restrict__ resid, const int32_t* __restrict__ rows,
                                    const float* __restrict__ norm_w, float eps,
                                    __nv_bfloat16* __restrict__ out, int64_t out_stride, int hidden,
                                    ClampParams cp) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float red[32];
  const int i = blockIdx.x;
  const float* rrow = resid + (int64_t)rows[i] * hidden;
  float ss = 0.f;
  for (int j = threadIdx.x; j < hidden; j += blockDim.x) ss += rrow[j] * rrow[j];
  const float inv = rsqrtf(block_sum(ss, red) / (float)hidden + eps);
  __nv_bfloat16* orow = out + (int64_t)i * out_stride;
  for (int j = threadIdx.x; j < hidden; j += blockDim.x)
    orow[j] = f_to_bf16(mu_clamp(norm_w[j] * (rrow[j] * inv), cp));
}

// ---------------------------------------------------------------------------
__global__ void reduce_clamp_kernel(const float* __restrict__ partials, int64_t partial_stride,
                                    int num_partials, float* __restrict__ dst,
                                    __nv_bfloat16* __restrict__ dst_bf16, int64_t dst_bf16_stride,
                                    int hidden, int64_t total, ClampParams cp) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < num_partials; ++p) s += partials[p * partial_stride + i];
    s = mu_clamp(s, cp);
    dst[i] = s;
    if (dst_bf16) {
      const int64_t t = i / hidden, j = i - t * hidden;
      dst_bf16[t * dst_bf16_stride + j] = f_to_bf16(s);
    }
  }
}

// out[t][c] = bf16(silu(sum_p partials[p][t][c] + bias[c])): the split-K
// tail of a narrow bias + SiLU projection (the INL controller's input layer).
__global__ void reduce_bias_silu_kernel(const float* __restrict__ partials, int64_t partial_stride,
                                        int num_partials, const float* __restrict__ bias,
                                        __nv_bfloat16* __restrict__ out, int64_t out_stride,
                                        int cols, int64_t total) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / cols;
    const int c = (int)(i - t * cols);
    float s = bias[c];
    for (int p = 0; p < num_partials; ++p) s += partials[p * partial_stride + i];
    out[t * out_stride + c] = f_to_bf16(silu(s));
  }
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
// torch.nn.functional.softplus with beta=1, threshold=20.
__device__ __forceinline__ float softplusf_(float x) { return x > 20.f ? x : log1pf(expf(x)); }

constexpr int kMaxExperts = 16;
constexpr int kInlMaxVecExperts = 8;  // the register-resident INL kernel routes over up to 8

__global__ void inl_dynamics_kernel(const float* __restrict__ h, const float* __restrict__ ctrl_raw,
                                    const float* __restrict__ ctrl_bias,
                                    const float* __restrict__ muproj,
                                    const float* __restrict__ mu_param, float dt, float* __restrict__ v,
                                    int v_zero, __nv_bfloat16* __restrict__ v_bf16,
                                    int64_t v_bf16_stride,
                                    float* __restrict__ resid, __nv_bfloat16* __restrict__ mu_out,
                                    int64_t mu_out_stride, const float* __restrict__ norm_w, float eps,
                                    __nv_bfloat16* __restrict__ norm_out, int64_t norm_out_stride,
                                    const int32_t* __restrict__ token_ids,
                                    const __nv_bfloat16* __restrict__ router_w, int num_experts,
                                    int vocab, int32_t* __restrict__ expert_ids, int hidden,
                                    ClampParams cp_norm) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  extern __shared__ float srow[];
  __shared__ float red[32];
  __shared__ float dots[kMaxExperts];
  const int t = blockIdx.x;
  const int64_t base = (int64_t)t * hidden;
  const float* crow = ctrl_raw + (int64_t)t * 3 * hidden;
  float ss = 0.f;
  float edot[kMaxExperts];
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) edot[e] = 0.f;
  for (int j = threadIdx.x; j < hidden; j += blockDim.x) {
    const float a = sigmoidf_(crow[j] + ctrl_bias[j]);
    const float b = fminf(softplusf_(crow[hidden + j] + ctrl_bias[hidden + j]), 2.f);
    const float g = sigmoidf_(crow[2 * hidden + j] + ctrl_bias[2 * hidden + j]);
    const float mu_c = mu_param[j] + muproj[base + j];
    const float hj = h[base + j];
    float vn = a * (v_zero ? 0.f : v[base + j]) - b * (hj - mu_c);
    vn = fminf(fmaxf(vn, -10.f), 10.f);
    const float hn = hj + dt * g * vn;
    const float r = resid[base + j] + hn;
    resid[base + j] = r;
    v[base + j] = vn;
    if (v_bf16) v_bf16[(int64_t)t * v_bf16_stride + j] = f_to_bf16(vn);
    if (mu_out) mu_out[(int64_t)t * mu_out_stride + j] = f_to_bf16(mu_c);
    srow[j] = r;
    ss += r * r;
    if (router_w) {
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e)
        if (e < num_experts) edot[e] += mu_c * bf16_to_f(router_w[(int64_t)e * hidden + j]);
    }
  }
  const float total = block_sum(ss, red);
  if (router_w) {
    for (int e = 0; e < num_experts; ++e) {
      const float d = block_sum(edot[e], red);
      if (threadIdx.x == 0) dots[e] = d;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int id = token_ids[t];
      id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
      const int base_e = id % num_experts;
      int best = 0;
      float bestv = -INFINITY;
      for (int e = 0; e < num_experts; ++e) {
        const float s = (e == base_e ? 10.f : 0.f) + dots[e];
        if (s > bestv) {
          bestv = s;
          best = e;
        }
      }
      expert_ids[t] = best;
    }
  }
  if (norm_out) {
    const float inv = rsqrtf(total / (float)hidden + eps);
    __nv_bfloat16* orow = norm_out + (int64_t)t * norm_out_stride;
    for (int j = threadIdx.x; j < hidden; j += blockDim.x)
      orow[j] = f_to_bf16(mu_clamp(norm_w[j] * (srow[j] * inv), cp_norm));
  }
}

// Register-resident INL step (same arithmetic as inl_dynamics_kernel):
// blockDim.x * VPT float4 = hidden; all loads of a chunk issued together.
// Per-row sums of the INL kernel: the squared residual and one router dot
// product per expert, reduced over the CTA together (one shared-memory pass
// for all of them instead of one per value).
template <int NV>
__device__ __forceinline__ void block_sums(float (&x)[NV], float* red /* [32][NV] */) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < NV; ++k) x[k] = warp_sum(x[k]);
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < NV; ++k) red[warp * NV + k] = x[k];
  __syncthreads();
  const int nw = blockDim.x >> 5;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += red[w * NV + k];  // same order in every thread
    x[k] = t;
  }
}

template <int VPT>
__global__ void __launch_bounds__(256, VPT <= 4 ? 3 : 1)
    inl_dynamics_vec_kernel(const float* __restrict__ h, const float* __restrict__ ctrl_raw,
                            const float* __restrict__ ctrl_bias, const float* __restrict__ muproj,
                            const float* __restrict__ mu_param, float dt, float* __restrict__ v,
                            int v_zero, __nv_bfloat16* __restrict__ v_bf16, int64_t v_bf16_stride,
                            float* __restrict__ resid, __nv_bfloat16* __restrict__ mu_out,
                            int64_t mu_out_stride, const float* __restrict__ norm_w, float eps,
                            __nv_bfloat16* __restrict__ norm_out, int64_t norm_out_stride,
                            const int32_t* __restrict__ token_ids,
                            const __nv_bfloat16* __restrict__ router_w, int num_experts, int vocab,
                            int32_t* __restrict__ expert_ids, int hidden, ClampParams cp_norm) {
  // programmatic dependent launch: let the next kernel launch once every CTA
  // of this one runs, and wait for the previous kernel before touching memory
  grid_dep_launch();
  grid_dep_wait();
  constexpr int NV = 1 + kInlMaxVecExperts;      // squared sum + router dots
  __shared__ float red[32 * NV];
  const int t = blockIdx.x;
  const int n = blockDim.x;
  const int64_t base4 = (int64_t)t * (hidden / 4);
  const int H4 = hidden / 4;
  const float4* h4 = reinterpret_cast<const float4*>(h) + base4;
  const float4* c4 = reinterpret_cast<const float4*>(ctrl_raw) + (int64_t)t * 3 * H4;
  const float4* b4 = reinterpret_cast<const float4*>(ctrl_bias);
  const float4* mp4 = reinterpret_cast<const float4*>(muproj) + base4;
  const float4* mu4 = reinterpret_cast<const float4*>(mu_param);
  float4* v4 = reinterpret_cast<float4*>(v) + base4;
  float4* r4 = reinterpret_cast<float4*>(resid) + base4;
  float acc[NV];
#pragma unroll
  for (int e = 0; e < NV; ++e) acc[e] = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int q = threadIdx.x + i * n;  // float4 index within the row
    const float4 ca = c4[q], cb = c4[H4 + q], cg = c4[2 * H4 + q];
    const float4 mpv = mp4[q], hv = h4[q], rv = r4[q];
    const float4 vv = v_zero ? make_float4(0.f, 0.f, 0.f, 0.f) : v4[q];
    const float4 ba = b4[q], bb = b4[H4 + q], bg = b4[2 * H4 + q], muv = mu4[q];
    const float cav[4] = {ca.x, ca.y, ca.z, ca.w}, cbv[4] = {cb.x, cb.y, cb.z, cb.w};
    const float cgv[4] = {cg.x, cg.y, cg.z, cg.w}, bav[4] = {ba.x, ba.y, ba.z, ba.w};
    const float bbv[4] = {bb.x, bb.y, bb.z, bb.w}, bgv[4] = {bg.x, bg.y, bg.z, bg.w};
    const float mpa[4] = {mpv.x, mpv.y, mpv.z, mpv.w}, mua[4] = {muv.x, muv.y, muv.z, muv.w};
    const float ha[4] = {hv.x, hv.y, hv.z, hv.w}, va[4] = {vv.x, vv.y, vv.z, vv.w};
    const float ra[4] = {rv.x, rv.y, rv.z, rv.w};
    float vn[4], rn[4], muc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float a = sigmoidf_(cav[u] + bav[u]);
      const float bta = fminf(softplusf_(cbv[u] + bbv[u]), 2.f);
      const float g = sigmoidf_(cgv[u] + bgv[u]);
      muc[u] = mua[u] + mpa[u];
      float x = a * va[u] - bta * (ha[u] - muc[u]);
      x = fminf(fmaxf(x, -10.f), 10.f);
      vn[u] = x;
      rn[u] = ra[u] + (ha[u] + dt * g * x);
      acc[0] += rn[u] * rn[u];
    }
    r4[q] = make_float4(rn[0], rn[1], rn[2], rn[3]);
    v4[q] = make_float4(vn[0], vn[1], vn[2], vn[3]);
    if (v_bf16) {
      uint2 o;
      o.x = pack_bf16x2(vn[0], vn[1]);
      o.y = pack_bf16x2(vn[2], vn[3]);
      *reinterpret_cast<uint2*>(v_bf16 + (int64_t)t * v_bf16_stride + 4 * q) = o;
    }
    if (mu_out) {
      uint2 o;
      o.x = pack_bf16x2(muc[0], muc[1]);
      o.y = pack_bf16x2(muc[2], muc[3]);
      *reinterpret_cast<uint2*>(mu_out + (int64_t)t * mu_out_stride + 4 * q) = o;
    }
    if (router_w) {
#pragma unroll
      for (int e = 0; e < kInlMaxVecExperts; ++e) {
        if (e < num_experts) {
          const uint2 w = *reinterpret_cast<const uint2*>(router_w + (int64_t)e * hidden + 4 * q);
          const float2 w01 = unpack_bf16x2(w.x), w23 = unpack_bf16x2(w.y);
          acc[1 + e] += muc[0] * w01.x + muc[1] * w01.y + muc[2] * w23.x + muc[3] * w23.y;
        }
      }
    }
  }
  block_sums<NV>(acc, red);
  if (router_w && threadIdx.x == 0) {
    int id = token_ids[t];
    id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
    const int base_e = id % num_experts;
    int best = 0;
    float bestv = -INFINITY;
#pragma unroll
    for (int e = 0; e < kInlMaxVecExperts; ++e) {
      if (e < num_experts) {
        const float sc = (e == base_e ? 10.f : 0.f) + acc[1 + e];
        if (sc > bestv) {
          bestv = sc;
          best = e;
        }
      }
    }
    expert_ids[t] = best;
  }
  if (norm_out) {
    // the row just written by this same thread comes back from L1
    const float inv = rsqrtf(acc[0] / (float)hidden + eps);
    const float4* w4 = reinterpret_cast<const float4*>(norm_w);
    uint2* orow = reinterpret_cast<uint2*>(norm_out + (int64_t)t * norm_out_stride);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int q = threadIdx.x + i * n;
      const float4 w = w4[q], r = r4[q];
      uint2 o;
      o.x = pack_bf16x2(mu_clamp(w.x * (r.x * inv), cp_norm), mu_clamp(w.y * (r.y * inv), cp_norm));
      o.y = pack_bf16x2(mu_clamp(w.z * (r.z * inv), cp_norm), mu_clamp(w.w * (r.w * inv), cp_norm));
      orow[q] = o;
    }
  }
}

}  // namespace muk

using namespace muk;

extern "C" int muk_embed(const int32_t* ids, const void* table, int64_t table_stride, float* resid,
                         int num_tokens, int hidden, int vocab, int clamp, float mu, float clamp_min,
                         float clamp_max, void* stream) {
  MUK_REQUIRE(num_tokens >= 0 && hidden > 0 && (hidden % 2) == 0 && vocab > 0,
              "muk_embed: bad shape T=%d H=%d V=%d", num_tokens, hidden, vocab);
  MUK_REQUIRE(ids && table && resid, "muk_embed: null pointer");
  MUK_REQUIRE(table_stride >= hidden && (table_stride % 2) == 0, "muk_embed: bad table stride");
  if (num_tokens == 0) return MUK_OK;
  embed_kernel<<<num_tokens, kRowThreads, 0, as_stream(stream)>>>(
      ids, reinterpret_cast<const __nv_bfloat16*>(table), table_stride, resid, hidden, vocab,
      make_clamp(clamp, mu, clamp_min, clamp_max));
  return check_launch("muk_embed");
}

template <typename DT>
static int launch_residual_rmsnorm(float* resid, const DT* partials, int64_t partial_stride,
                                   int64_t partial_row_stride, int num_partials,
                                   const int32_t* delta_rows, const float* norm_w, float eps,
                                   void* out, int64_t out_stride, int num_tokens, int hidden,
                                   int clamp_delta, int clamp_sum, int clamp_norm, float mu,
                                   float clamp_min, float clamp_max, void* stream,
                                   const char* name) {
  MUK_REQUIRE(num_tokens >= 0 && hidden > 0 && hidden % 4 == 0 && hidden <= kMaxHidden,
              "%s: hidden=%d must be a multiple of 4 and <= %d", name, hidden, kMaxHidden);
  MUK_REQUIRE(resid != nullptr && MUK_ALIGNED16(resid), "%s: resid", name);
  MUK_REQUIRE(num_partials >= 0 && (num_partials == 0 || (partials && MUK_ALIGNED16(partials) &&
                                                          partial_row_stride % 4 == 0 &&
                                                          partial_stride % 4 == 0)),
              "%s: partials must be 16-byte aligned rows", name);
  MUK_REQUIRE(out == nullptr || (norm_w && out_stride >= hidden && out_stride % 2 == 0),
              "%s: out needs norm_w and an even stride >= hidden", name);
  if (num_tokens == 0) return MUK_OK;
  ClampParams cp = make_clamp(1, mu, clamp_min, clamp_max);
  const ClampParams cpn = make_clamp(clamp_norm, mu, clamp_min, clamp_max);
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
  const int vpt = row_vpt(hidden);
  const bool vec_ok = vpt != 0 && MUK_ALIGNED16(norm_w) && out_stride % 4 == 0 &&
                      (partial_row_stride % 4 == 0) && (out == nullptr || ((uintptr_t)out & 7) == 0);
  cudaStream_t st = as_stream(stream);
#define MUK_RRN(V, THREADS)                                                                     \
  launch_pdl(residual_rmsnorm_vec_kernel<V, DT>,                                                   \
      dim3(num_tokens), dim3(THREADS), 0, st,                                                      \
      resid, partials, partial_stride, partial_row_stride, num_partials, delta_rows, norm_w, eps, \
      o, out_stride, hidden, clamp_delta, clamp_sum, cpn, cp)
  bool done = false;
  if (vec_ok) {
    done = true;
    switch (vpt) {
      case -1: MUK_RRN(1, hidden / 4); break;
      case 1: MUK_RRN(1, 256); break;
      case 2: MUK_RRN(2, 256); break;
      case 4: MUK_RRN(4, 256); break;
      case 8: MUK_RRN(8, 256); break;
      case 16: MUK_RRN(16, 256); break;
      default: done = false;
    }
  }
  if (!done)
    launch_pdl(residual_rmsnorm_kernel<DT>,
               dim3(num_tokens), dim3(kRowThreads), hidden * sizeof(float), st,
        resid, partials, partial_stride, partial_row_stride, num_partials, delta_rows, norm_w, eps,
        o, out_stride, hidden, clamp_delta, clamp_sum, cpn, cp);
#undef MUK_RRN
  return check_launch(name);
}

extern "C" int muk_residual_rmsnorm(float* resid, const float* partials, int64_t partial_stride,
                                    int64_t partial_row_stride, int num_partials,
                                    const int32_t* delta_rows, const float* norm_w, float eps,
                                    void* out, int64_t out_stride, int num_tokens, int hidden,
                                    int clamp_delta, int clamp_sum, int clamp_norm, float mu,
                                    float clamp_min, float clamp_max, void* stream) {
  return launch_residual_rmsnorm<float>(resid, partials, partial_stride, partial_row_stride,
                                        num_partials, delta_rows, norm_w, eps, out, out_stride,
                                        num_tokens, hidden, clamp_delta, clamp_sum, clamp_norm, mu,
                                        clamp_min, clamp_max, stream, "muk_residual_rmsnorm");
}

extern "C" int muk_residual_rmsnorm_bf16(float* resid, const void* delta, int64_t delta_row_stride,
                                         const int32_t* delta_rows, const float* norm_w, float eps,
                                         void* out, int64_t out_stride, int num_tokens, int hidden,
                                         int clamp_delta, int clamp_sum, int clamp_norm, float mu,
                                         float clamp_min, float clamp_max, void* stream) {
  MUK_REQUIRE(delta != nullptr, "muk_residual_rmsnorm_bf16: delta is null");
  return launch_residual_rmsnorm<__nv_bfloat16>(
      resid, reinterpret_cast<const __nv_bfloat16*>(delta), 0, delta_row_stride, 1, delta_rows,
      norm_w, eps, out, out_stride, num_tokens, hidden, clamp_delta, clamp_sum, clamp_norm, mu,
      clamp_min, clamp_max, stream, "muk_residual_rmsnorm_bf16");
}

extern "C" int muk_rmsnorm_rows(const float* resid, const int32_t* rows, int num_rows,
                                const float* norm_w, float eps, void* out, int64_t out_stride,
                                int hidden, int clamp, float mu, float clamp_min, float clamp_max,
                                void* stream) {
  MUK_REQUIRE(resid && rows && norm_w && out && hidden > 0 && out_stride >= hidden,
              "muk_rmsnorm_rows: bad arguments");
  if (num_rows <= 0) return MUK_OK;
  launch_pdl(rmsnorm_rows_kernel, dim3(num_rows), dim3(kRowThreads), 0, as_stream(stream),
      resid, rows, norm_w, eps, reinterpret_cast<__nv_bfloat16*>(out), out_stride, hidden,
      make_clamp(clamp, mu, clamp_min, clamp_max));
  return check_launch("muk_rmsnorm_rows");
}

extern "C" int muk_reduce_clamp(const float* partials, int64_t partial_stride, int num_partials,
                                float* dst_f32, void* dst_bf16, int64_t dst_bf16_stride,
                                int num_tokens, int hidden, int clamp, float mu, float clamp_min,
                                float clamp_max, void* stream) {
  MUK_REQUIRE(partials && dst_f32 && num_partials >= 1 && hidden > 0,
              "muk_reduce_clamp: bad arguments");
  MUK_REQUIRE(dst_bf16 == nullptr || dst_bf16_stride >= hidden, "muk_reduce_clamp: bad stride");
  const int64_t total = (int64_t)num_tokens * hidden;
  if (total == 0) return MUK_OK;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(reduce_clamp_kernel, dim3(blocks), dim3(256), 0, as_stream(stream),
      partials, partial_stride, num_partials, dst_f32, reinterpret_cast<__nv_bfloat16*>(dst_bf16),
      dst_bf16_stride, hidden, total, make_clamp(clamp, mu, clamp_min, clamp_max));
  return check_launch("muk_reduce_clamp");
}

extern "C" int muk_reduce_bias_silu(const float* partials, int64_t partial_stride,
                                    int num_partials, const float* bias, void* out,
                                    int64_t out_stride, int rows, int cols, void* stream) {
  MUK_REQUIRE(partials && bias && out && num_partials >= 1 && rows >= 0 && cols > 0 &&
                  out_stride >= cols && (num_partials == 1 || partial_stride >= (int64_t)rows * cols),
              "muk_reduce_bias_silu: bad arguments (rows %d cols %d partials %d)", rows, cols,
              num_partials);
  if (rows == 0) return MUK_OK;
  const int64_t total = (int64_t)rows * cols;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 4 * 148) blocks = 4 * 148;
  launch_pdl(reduce_bias_silu_kernel, dim3(blocks), dim3(256), 0, as_stream(stream),
      partials, partial_stride, num_partials, bias, reinterpret_cast<__nv_bfloat16*>(out),
      out_stride, cols, total);
  return check_launch("muk_reduce_bias_silu");
}

extern "C" int muk_inl_dynamics(const float* h, const float* ctrl_raw, const float* ctrl_bias,
                                const float* muproj, const float* mu_param, float dt, float* v,
                                int v_zero, void* v_bf16, int64_t v_bf16_stride, float* resid,
                                void* mu_out,
                                int64_t mu_out_stride, const float* norm_w, float eps,
                                void* norm_out, int64_t norm_out_stride, const int32_t* token_ids,
                                const void* router_w, int num_experts, int vocab,
                                int32_t* expert_ids, int num_tokens, int hidden, int clamp_norm,
                                float mu, float clamp_min, float clamp_max, void* stream) {
  MUK_REQUIRE(h && ctrl_raw && ctrl_bias && muproj && mu_param && v && resid,
              "muk_inl_dynamics: null pointer");
  MUK_REQUIRE(hidden > 0 && hidden <= kMaxHidden, "muk_inl_dynamics: hidden=%d", hidden);
  MUK_REQUIRE(norm_out == nullptr || norm_w, "muk_inl_dynamics: norm_out needs norm_w");
  MUK_REQUIRE(router_w == nullptr ||
                  (token_ids && expert_ids && num_experts >= 1 && num_experts <= kMaxExperts &&
                   vocab > 0),
              "muk_inl_dynamics: routing needs token_ids, expert_ids and 1..%d experts",
              kMaxExperts);
  if (num_tokens == 0) return MUK_OK;
  cudaStream_t st = as_stream(stream);
  const ClampParams cpn = make_clamp(clamp_norm, mu, clamp_min, clamp_max);
  __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(v_bf16);
  __nv_bfloat16* mo = reinterpret_cast<__nv_bfloat16*>(mu_out);
  __nv_bfloat16* no = reinterpret_cast<__nv_bfloat16*>(norm_out);
  const __nv_bfloat16* rw = reinterpret_cast<const __nv_bfloat16*>(router_w);
  const int vpt = row_vpt(hidden);
  const bool vec_ok = vpt != 0 && MUK_ALIGNED16(h) && MUK_ALIGNED16(ctrl_raw) &&
                      MUK_ALIGNED16(ctrl_bias) && MUK_ALIGNED16(muproj) &&
                      MUK_ALIGNED16(mu_param) && MUK_ALIGNED16(v) && MUK_ALIGNED16(resid) &&
                      (norm_out == nullptr || (MUK_ALIGNED16(norm_w) && norm_out_stride % 4 == 0 &&
                                               ((uintptr_t)norm_out & 7) == 0)) &&
                      (v_bf16 == nullptr || (v_bf16_stride % 4 == 0 && ((uintptr_t)v_bf16 & 7) == 0)) &&
                      (mu_out == nullptr || (mu_out_stride % 4 == 0 && ((uintptr_t)mu_out & 7) == 0)) &&
                      (router_w == nullptr || ((uintptr_t)router_w & 7) == 0);
#define MUK_INL(V, THREADS)                                                                      \
  launch_pdl(inl_dynamics_vec_kernel<V>,                                                           \
      dim3(num_tokens), dim3(THREADS), 0, st,                                                      \
      h, ctrl_raw, ctrl_bias, muproj, mu_param, dt, v, v_zero, vb, v_bf16_stride, resid, mo,            \
      mu_out_stride, norm_w, eps, no, norm_out_stride, token_ids, rw, num_experts, vocab,        \
      expert_ids, hidden, cpn)
  if (router_w != nullptr && num_experts > kInlMaxVecExperts) {
    launch_pdl(inl_dynamics_kernel, dim3(num_tokens), dim3(kRowThreads), hidden * sizeof(float), st,
        h, ctrl_raw, ctrl_bias, muproj, mu_param, dt, v, v_zero, vb, v_bf16_stride, resid, mo,
        mu_out_stride, norm_w, eps, no, norm_out_stride, token_ids, rw, num_experts, vocab,
        expert_ids, hidden, cpn);
  } else if (vec_ok && vpt == -1) {
    MUK_INL(1, hidden / 4);
  } else if (vec_ok && vpt == 1) {
    MUK_INL(1, 256);
  } else if (vec_ok && vpt == 2) {
    MUK_INL(2, 256);
  } else if (vec_ok && vpt == 4) {
    MUK_INL(4, 256);
  } else {
    launch_pdl(inl_dynamics_kernel, dim3(num_tokens), dim3(kRowThreads), hidden * sizeof(float), st,
        h, ctrl_raw, ctrl_bias, muproj, mu_param, dt, v, v_zero, vb, v_bf16_stride, resid, mo,
        mu_out_stride, norm_w, eps, no, norm_out_stride, token_ids, rw, num_experts, vocab,
        expert_ids, hidden, cpn);
  }
#undef MUK_INL
  return check_launch("muk_inl_dynamics");
}
