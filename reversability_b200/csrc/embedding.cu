// Token + learned position embedding, forward and backward (replaces
// nn.Embedding lookups at model.py:101 / reversible.py:106 and their autograd
// backward, including the tied-weight accumulation of the head gradient).
//
// Forward: x[r] = tok[ids[r]] + pos[r % T], one warp per row, 16-byte loads.
// Backward, deterministic (no floating-point atomics):
//   1. rows are sorted by token id with a stable radix sort (CUB, keys = ids,
//      values = row indices), so equal ids become contiguous runs in row order;
//   2. each run is summed in two fixed-order passes (per-32-row pieces, then
//      the pieces of a run in order, one warp per run) and added into g_tok[id];
//   3. one thread per (position t, 4 columns) sums dx[b*T + t] over b in
//      order into g_pos[t].
// Step 1 depends on the ids alone: rk_embedding_bwd_sort runs it by itself
// (a caller can issue it early, on another stream) and
// rk_embedding_bwd_sorted runs steps 2 and 3 from its result;
// rk_embedding_bwd is the two in sequence.
// The row cotangent is dx (+ dx2 when given: the boundary state p = q = x of
// the reversible stack receives one cotangent through each).
// Ids outside [0, V) set RK_DEV_EMB_INDEX and contribute nothing.
#include <cub/cub.cuh>
#include "vec.cuh"

namespace rk {

__global__ void __launch_bounds__(256) emb_fwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ tok,
                                                      const float* __restrict__ pos, float* __restrict__ out,
                                                      int64_t rows, int T, int d, int64_t V, unsigned int* status) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int64_t id = ids[r];
  const bool ok = id >= 0 && id < V;
  if (!ok && lane == 0) flag_error(status, RK_DEV_EMB_INDEX);
  const float* tr = tok + (ok ? id : 0) * d;
  const float* pr = pos + (r % T) * d;
  float* orow = out + r * d;
  for (int c = lane * 4; c < d; c += 128) {
    float a[4], b[4], o[4];
    load_vec<float, 4>(tr + c, a);
    load_vec<float, 4>(pr + c, b);
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = (ok ? a[e] : 0.f) + b[e];
    store_vec<float, 4>(orow + c, o);
  }
}

// Sort keys (ids outside [0, V) become V, a run the backward skips) and row indices.
__global__ void keys_kernel(const int64_t* __restrict__ ids, int64_t* __restrict__ keys, int* __restrict__ rows_out,
                            int64_t n, int64_t V) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const int64_t id = ids[i];
    keys[i] = (id >= 0 && id < V) ? id : V;
    rows_out[i] = (int)i;
  }
}

// Token-gradient reduction in two fixed-order passes over the sorted rows.
// Pass 1: warp w owns sorted positions [32r, 32r+32) and 128-column chunk c
// (w = r * chunks + c); it sums the rows of each run piece inside its range in
// position order (one 16-byte vector per lane per row, eight row loads in
// flight) and writes the piece's sum at piece[start of the piece]. Pass 2: the CTA of each run start adds the pieces
// of its run (one per 32-row range it overlaps) in range order into g_tok.
// Every sum has a fixed order, so g_tok is bitwise reproducible, and a long
// run (a frequent token) is read by many warps in parallel.
__global__ void __launch_bounds__(256) emb_tok_piece_kernel(const int64_t* __restrict__ skeys,
                                                            const int* __restrict__ srows,
                                                            const float* __restrict__ dx,
                                                            const float* __restrict__ dx2, float* __restrict__ piece,
                                                            int64_t rows, int d) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int lane = threadIdx.x & 31;
  // warp gw: 32-row range gw / nch, 128-column chunk gw % nch
  const int nch = (d + 127) / 128;
  const int64_t gw = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t r0 = gw / nch * 32;
  if (r0 >= rows) return;
  const int n = (int)(r0 + 32 < rows ? 32 : rows - r0);
  // the warp's sorted rows and run ends, one per lane; every row load is
  // issued ahead of its add (eight in flight), the adds stay in row order
  const int my_row = lane < n ? srows[r0 + lane] : 0;
  const int64_t my_key = lane < n ? skeys[r0 + lane] : 0;
  const int64_t next_key = lane + 1 < n ? skeys[r0 + lane + 1] : my_key;
  const unsigned run_end = __ballot_sync(0xffffffffu, lane < n && (lane + 1 == n || next_key != my_key));
  {
    const int c = (int)(gw % nch) * 128 + lane * 4;
    int start = 0;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < n; j0 += 8) {
      float v[8][4];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int row = __shfl_sync(0xffffffffu, my_row, (j0 + u) & 31);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[u][e] = 0.f;
        if (j0 + u < n && c < d) {
          const int64_t off = (int64_t)row * d + c;
          load_vec<float, 4>(dx + off, v[u]);
          if (dx2) {
            float v2[4];
            load_vec<float, 4>(dx2 + off, v2);
#pragma unroll
            for (int e = 0; e < 4; ++e) v[u][e] += v2[e];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        if (j < n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[e] += v[u][e];
          if ((run_end >> j) & 1u) {
            if (c < d) store_vec<float, 4>(piece + (r0 + start) * d + c, acc);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] = 0.f;
            start = j + 1;
          }
        }
      }
    }
  }
}

// Pass 2: the warp of each run start (one warp per sorted position) adds the
// pieces of its run, one per 32-row range it overlaps, in range order into
// g_tok; each lane owns 4 consecutive columns per step (16-byte piece loads,
// eight pieces in flight).
__global__ void __launch_bounds__(256) emb_tok_bwd_kernel(const int64_t* __restrict__ skeys,
                                                          const float* __restrict__ piece, float* __restrict__ g_tok,
                                                          int64_t rows, int d, int64_t V, unsigned int* status) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (i >= rows) return;
  const int64_t id = skeys[i];
  if (i > 0 && skeys[i - 1] == id) return;
  if (id < 0 || id >= V) {
    if (lane == 0) flag_error(status, RK_DEV_EMB_INDEX);
    return;
  }
  int64_t lo = i + 1, hi = rows;  // run end: first index with a different key
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (skeys[mid] == id) lo = mid + 1; else hi = mid;
  }
  const int64_t end = lo;
  for (int c = lane * 4; c < d; c += 128) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    int64_t p = i;
    while (p < end) {
      float t[8][4];
      int cnt = 0;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
#pragma unroll
        for (int e = 0; e < 4; ++e) t[u][e] = 0.f;
        if (p < end) {
          load_vec<float, 4>(piece + p * d + c, t[u]);
          p = (p / 32 + 1) * 32;
          ++cnt;
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < cnt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) s[e] += t[u][e];
        }
    }
    float* g = g_tok + id * d + c;
#pragma unroll
    for (int e = 0; e < 4; ++e) g[e] += s[e];
  }
}

// g_pos[t] += sum over b of dx[b*T + t] (+ dx2), in b order; one thread per
// (position, 4 columns), eight rows in flight.
__global__ void __launch_bounds__(256) emb_pos_bwd_kernel(const float* __restrict__ dx, const float* __restrict__ dx2,
                                                          float* __restrict__ g_pos, int64_t rows, int T, int d) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int q = d / 4;
  const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (item >= (int64_t)T * q) return;
  const int t = (int)(item / q), c = (int)(item % q) * 4;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t r0 = t; r0 < rows; r0 += 8 * (int64_t)T) {
    float v[8][4];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t r = r0 + u * (int64_t)T;
#pragma unroll
      for (int e = 0; e < 4; ++e) v[u][e] = 0.f;
      if (r < rows) {
        load_vec<float, 4>(dx + r * d + c, v[u]);
        if (dx2) {
          float v2[4];
          load_vec<float, 4>(dx2 + r * d + c, v2);
#pragma unroll
          for (int e = 0; e < 4; ++e) v[u][e] = v[u][e] + v2[e];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (r0 + u * (int64_t)T < rows) {
#pragma unroll
        for (int e = 0; e < 4; ++e) s[e] += v[u][e];
      }
  }
  float* g = g_pos + (int64_t)t * d + c;
#pragma unroll
  for (int e = 0; e < 4; ++e) g[e] += s[e];
}

}  // namespace rk

using namespace rk;

namespace {
int key_bits(int64_t V) {
  int b = 1;
  while (b < 63 && (1ll << b) < V) ++b;
  return b;
}
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
constexpr int64_t kMaxEmbWidth = 1024;  // widest embedding the piece buffer is sized for
size_t cub_temp_bytes(int64_t rows, int64_t V) {
  size_t temp = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, temp, (const int64_t*)nullptr, (int64_t*)nullptr, (const int*)nullptr,
                                  (int*)nullptr, (int)rows, 0, key_bits(V + 1));
  return temp;
}
}  // namespace

extern "C" int rk_embedding_fwd(const int64_t* ids, const float* tok, const float* pos, float* out, int64_t rows,
                                int64_t T, int64_t d, int64_t V, void* stream) {
  if (!ids || !tok || !pos || !out || rows < 0 || T <= 0 || d <= 0 || V <= 0) return RK_ERR_ARG;
  if (d % 4 || !rk_host::aligned(tok, 16) || !rk_host::aligned(pos, 16) || !rk_host::aligned(out, 16))
    return RK_ERR_ALIGN;
  if (rows == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rk_host::launch_k(emb_fwd_kernel, (unsigned)((rows + 7) / 8), 256, 0, s, ids, tok, pos, out, rows, (int)T, (int)d, V,
                                                            rk_host::device_status_ptr());
  return rk_host::launch_status();
}

namespace {
// The sort results lead the buffer (read by the second phase); the unsorted
// keys, row indices and the sort's temporary storage follow.
struct SortLayout {
  int64_t* skeys;
  int* srows;
  int64_t* keys;
  int* rows_in;
  void* temp;
  size_t temp_bytes;
};
size_t sort_bytes(int64_t rows, int64_t V) {
  return 2 * align256(rows * sizeof(int64_t)) + 2 * align256(rows * sizeof(int)) + align256(cub_temp_bytes(rows, V));
}
SortLayout sort_layout(void* buf, int64_t rows, int64_t V) {
  uint8_t* w = static_cast<uint8_t*>(buf);
  SortLayout l;
  l.skeys = reinterpret_cast<int64_t*>(w);
  w += align256(rows * sizeof(int64_t));
  l.srows = reinterpret_cast<int*>(w);
  w += align256(rows * sizeof(int));
  l.keys = reinterpret_cast<int64_t*>(w);
  w += align256(rows * sizeof(int64_t));
  l.rows_in = reinterpret_cast<int*>(w);
  w += align256(rows * sizeof(int));
  l.temp = w;
  l.temp_bytes = cub_temp_bytes(rows, V);
  return l;
}
}  // namespace

extern "C" int64_t rk_embedding_bwd_sort_bytes(int64_t rows, int64_t V) {
  if (rows <= 0 || V <= 0 || rows >= (1ll << 31)) return 0;
  return (int64_t)sort_bytes(rows, V);
}

extern "C" int rk_embedding_bwd_sort(const int64_t* ids, int64_t rows, int64_t V, void* sorted, int64_t sorted_bytes,
                                     void* stream) {
  if (!ids || rows < 0 || V <= 0 || rows >= (1ll << 31)) return RK_ERR_ARG;
  if (rows == 0) return RK_OK;
  if (!sorted || sorted_bytes < rk_embedding_bwd_sort_bytes(rows, V)) return RK_ERR_WORKSPACE;
  if (!rk_host::aligned(sorted, 16)) return RK_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SortLayout l = sort_layout(sorted, rows, V);
  rk_host::launch_k(keys_kernel, (unsigned)((rows + 255) / 256), 256, 0, s, ids, l.keys, l.rows_in, rows, V);
  int st = rk_host::launch_status();
  if (st) return st;
  size_t temp = l.temp_bytes;
  if (cub::DeviceRadixSort::SortPairs(l.temp, temp, l.keys, l.skeys, l.rows_in, l.srows, (int)rows, 0,
                                      key_bits(V + 1), s) != cudaSuccess)
    return RK_ERR_LAUNCH;
  rk_host::count_launch();
  return RK_OK;
}

extern "C" int64_t rk_embedding_bwd_sorted_workspace(int64_t rows, int64_t d) {
  if (rows <= 0 || d <= 0) return 0;
  return (int64_t)align256(rows * 4 * (size_t)d);
}

extern "C" int rk_embedding_bwd_sorted(const void* sorted, int64_t sorted_bytes, const float* dx, const float* dx2,
                                       float* g_tok, float* g_pos, int64_t rows, int64_t T, int64_t d, int64_t V,
                                       void* workspace, int64_t workspace_bytes, void* stream) {
  if (!dx || !g_tok || !g_pos || rows < 0 || T <= 0 || d <= 0 || V <= 0 || rows >= (1ll << 31)) return RK_ERR_ARG;
  if (d > kMaxEmbWidth) return RK_ERR_UNSUPPORTED;
  if (d % 4 || !rk_host::aligned(dx, 16) || (dx2 && !rk_host::aligned(dx2, 16))) return RK_ERR_ALIGN;
  if (rows == 0) return RK_OK;
  if (!sorted || sorted_bytes < rk_embedding_bwd_sort_bytes(rows, V)) return RK_ERR_WORKSPACE;
  if (!workspace || workspace_bytes < rk_embedding_bwd_sorted_workspace(rows, d)) return RK_ERR_WORKSPACE;
  if (!rk_host::aligned(sorted, 16) || !rk_host::aligned(workspace, 16)) return RK_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SortLayout l = sort_layout(const_cast<void*>(sorted), rows, V);
  float* piece = static_cast<float*>(workspace);
  const int64_t piece_warps = (rows + 31) / 32 * ((d + 127) / 128);
  rk_host::launch_k(emb_tok_piece_kernel, (unsigned)((piece_warps + 7) / 8), 256, 0, s, l.skeys, l.srows, dx, dx2,
                    piece, rows, (int)d);
  int st = rk_host::launch_status();
  if (st) return st;
  rk_host::launch_k(emb_tok_bwd_kernel, (unsigned)((rows + 7) / 8), 256, 0, s, l.skeys, piece, g_tok, rows, (int)d, V,
                    rk_host::device_status_ptr());
  st = rk_host::launch_status();
  if (st) return st;
  const int64_t items = T * (d / 4);
  rk_host::launch_k(emb_pos_bwd_kernel, (unsigned)((items + 255) / 256), 256, 0, s, dx, dx2, g_pos, rows, (int)T,
                    (int)d);
  return rk_host::launch_status();
}

extern "C" int64_t rk_embedding_bwd_workspace(int64_t rows, int64_t V) {
  if (rows <= 0 || V <= 0 || rows >= (1ll << 31)) return 0;
  return (int64_t)(sort_bytes(rows, V) + align256(rows * 4 * (size_t)kMaxEmbWidth));
}

extern "C" int rk_embedding_bwd(const int64_t* ids, const float* dx, const float* dx2, float* g_tok, float* g_pos,
                                int64_t rows, int64_t T, int64_t d, int64_t V, void* workspace, int64_t workspace_bytes,
                                void* stream) {
  if (!ids || !dx || !g_tok || !g_pos || rows < 0 || T <= 0 || d <= 0 || V <= 0 || rows >= (1ll << 31))
    return RK_ERR_ARG;
  if (d > kMaxEmbWidth) return RK_ERR_UNSUPPORTED;
  if (d % 4 || !rk_host::aligned(dx, 16) || (dx2 && !rk_host::aligned(dx2, 16))) return RK_ERR_ALIGN;
  if (rows == 0) return RK_OK;
  if (!workspace || workspace_bytes < rk_embedding_bwd_workspace(rows, V)) return RK_ERR_WORKSPACE;
  if (!rk_host::aligned(workspace, 16)) return RK_ERR_ALIGN;
  const int64_t sb = (int64_t)sort_bytes(rows, V);
  int st = rk_embedding_bwd_sort(ids, rows, V, workspace, sb, stream);
  if (st) return st;
  return rk_embedding_bwd_sorted(workspace, sb, dx, dx2, g_tok, g_pos, rows, T, d, V,
                                 static_cast<uint8_t*>(workspace) + sb, workspace_bytes - sb, stream);
}
