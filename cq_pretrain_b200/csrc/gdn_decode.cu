// One decode step of the gated delta rule for every head, fused into one kernel (CQ cached
// text decoding: one committed content token plus read-only query rows per step).
//
// Per head h with the fp32 state S [Dk, Dv] (updated in place):
//   k^ = k / ||k||,  q^_b = q_b / ||q_b|| * Dk^-1/2           (L2 norm with eps 1e-6 under the root)
//   S  = e^{g} S;   r = v - S^T k^;   S += k^ (beta r)^T;   y_b = S^T q^_b   (b over the query rows)
// Grid (H, Dv / 32), 128 threads: thread (warp w, lane l) owns column v0 + l and rows 32w..32w+31,
// so every state element is read and written once, with 32 consecutive floats per warp access.
// (Reference semantics: ops/gated_delta_net.py:315-352, the fused recurrent step.)
#include "common.cuh"

namespace cqb {

namespace {

constexpr int DK_DEC = 128, COLS = 32, DEC_THREADS = 128, MAX_ROWS = 4;

__global__ void __launch_bounds__(DEC_THREADS) gdn_decode_kernel(float* __restrict__ state, const float* __restrict__ q,
                                                                 const float* __restrict__ k,
                                                                 const float* __restrict__ v,
                                                                 const float* __restrict__ g,
                                                                 const float* __restrict__ beta,
                                                                 float* __restrict__ out, int H, int Dv, int rows) {
  __shared__ float kh[DK_DEC];
  __shared__ float qh[MAX_ROWS][DK_DEC];
  __shared__ float red[MAX_ROWS + 1][4][COLS];
  __shared__ float norms[MAX_ROWS + 1][4];
  const int h = blockIdx.x, v0 = blockIdx.y * COLS;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  // normalised k and q rows of this head (thread tid owns element tid)
  const float kv = k[(size_t)h * DK_DEC + tid];
  float sq = warp_sum(kv * kv);
  if (lane == 0) norms[0][w] = sq;
  float qv[MAX_ROWS];
  for (int b = 0; b < rows; ++b) {
    qv[b] = q[((size_t)b * H + h) * DK_DEC + tid];
    const float s = warp_sum(qv[b] * qv[b]);
    if (lane == 0) norms[b + 1][w] = s;
  }
  __syncthreads();
  const float kscale = rsqrtf(norms[0][0] + norms[0][1] + norms[0][2] + norms[0][3] + 1e-6f);
  kh[tid] = kv * kscale;
  for (int b = 0; b < rows; ++b)
    qh[b][tid] = qv[b] * rsqrtf(norms[b + 1][0] + norms[b + 1][1] + norms[b + 1][2] + norms[b + 1][3] + 1e-6f) *
                 rsqrtf((float)DK_DEC);
  __syncthreads();
  // decayed state column, partial S^T k^ over this thread's 32 rows
  const float decay = __expf(g[h]);
  float* col = state + ((size_t)h * DK_DEC + w * 32) * Dv + v0 + lane;
  float s[32];
  float dot = 0.f;
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    s[r] = col[(size_t)r * Dv] * decay;
    dot += s[r] * kh[w * 32 + r];
  }
  red[0][w][lane] = dot;
  __syncthreads();
  const float total = red[0][0][lane] + red[0][1][lane] + red[0][2][lane] + red[0][3][lane];
  const float rb = (v[(size_t)h * Dv + v0 + lane] - total) * beta[h];
  float y[MAX_ROWS] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    s[r] += kh[w * 32 + r] * rb;
    col[(size_t)r * Dv] = s[r];
    for (int b = 0; b < rows; ++b) y[b] += s[r] * qh[b][w * 32 + r];
  }
  for (int b = 0; b < rows; ++b) red[b + 1][w][lane] = y[b];
  __syncthreads();
  if (w == 0)
    for (int b = 0; b < rows; ++b)
      out[((size_t)b * H + h) * Dv + v0 + lane] =
          red[b + 1][0][lane] + red[b + 1][1][lane] + red[b + 1][2][lane] + red[b + 1][3][lane];
}

}  // namespace

// state fp32 [H, 128, Dv] (in place); q fp32 [rows, H, 128] (rows <= 4); k fp32 [H, 128];
// v fp32 [H, Dv]; g, beta fp32 [H]; out fp32 [rows, H, Dv].
void gdn_decode_step(at::Tensor state, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta,
                     at::Tensor out) {
  for (auto* t : {&state, &q, &k, &v, &g, &beta, &out})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous(),
                "gdn_decode_step: contiguous fp32 CUDA tensors");
  TORCH_CHECK(state.dim() == 3 && state.size(1) == DK_DEC && state.size(2) % COLS == 0,
              "state must be [H, 128, Dv] with Dv a multiple of 32");
  const int H = state.size(0), Dv = state.size(2), rows = q.size(0);
  TORCH_CHECK(rows >= 1 && rows <= MAX_ROWS && q.numel() == (int64_t)rows * H * DK_DEC, "q must be [rows<=4, H, 128]");
  TORCH_CHECK(k.numel() == (int64_t)H * DK_DEC && v.numel() == (int64_t)H * Dv && g.numel() == H &&
                  beta.numel() == H && out.numel() == (int64_t)rows * H * Dv,
              "gdn_decode_step: shapes");
  gdn_decode_kernel<<<dim3(H, Dv / COLS), DEC_THREADS, 0, stream()>>>(
      state.data_ptr<float>(), q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), g.data_ptr<float>(),
      beta.data_ptr<float>(), out.data_ptr<float>(), H, Dv, rows);
  CQB_LAUNCH_CHECK();
  count_launch();
}

}  // namespace cqb
