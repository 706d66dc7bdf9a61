// Sparse per-leaf histograms (fixed-point modes).
//
// The reference builds the histograms of a sparse matrix from its stored
// entries only (gpu_sparse.mojo:525, _sparse_hist_kernel): a feature's
// implicit entries all fall in one bin, whose cell is the leaf total minus the
// feature's other bins.  Here every feature f gets such a default bin d_f (its
// most frequent bin over the training rows, found on the device) and every
// row the list of its entries whose bin is not d_f, packed f << 8 | bin in
// row-major CSR order.  A warp takes one row at a time and adds the row's
// gradient to the cells of its listed entries only; the default bins are
// filled in from the segment's totals before the cells leave shared memory,
// so the work slot is cell for cell what the dense kernel writes (integer
// sums, any order) and the split scan is unchanged.
//
// For configs[2] (400 numeric columns 90% zero plus 8 categorical, 63 bins)
// a row lists ~50 of its 408 bins: the histogram reads ~200 B a row instead of
// 416 and issues ~100 shared atomics instead of 816.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "gbdt_device.cuh"
#include "gbdt_kernels.cuh"

namespace mtb {
namespace {

constexpr int kSparseThreads = 1024;
constexpr int kSparseUnroll = 4;  // rows whose entries a warp loads at once

// Shared-memory words of the sparse cells: planes x F x BP (BP = bins
// rounded up to a power of two; cell (f, b) of a plane is word
// f * BP + ((b + f) & (BP - 1)), the rotation spreading the cells a warp's
// entries hit over the banks).
__host__ __device__ inline size_t sparse_hist_words(int planes, int F, int BP) {
  return (size_t)planes * F * BP;
}
__host__ __device__ inline size_t sparse_hist_smem(int planes, int F, int BP) {
  return sparse_hist_words(planes, F, BP) * 4 + kHistBatchSmem + 64;
}

// d_f: the most frequent bin of every feature over all rows (lowest bin on
// ties).  One block per feature.
__global__ void __launch_bounds__(256) k_sparse_default_bins(const uint8_t* __restrict__ bins_cm, long long n,
                                                            int* __restrict__ default_bin) {
  __shared__ unsigned int cnt[256];
  for (int b = threadIdx.x; b < 256; b += blockDim.x) cnt[b] = 0u;
  __syncthreads();
  const uint8_t* col = bins_cm + (long long)blockIdx.x * n;
  const long long n16 = ((uintptr_t)col & 15) == 0 ? n / 16 : 0;
  const uint4* col4 = reinterpret_cast<const uint4*>(col);
  for (long long i = threadIdx.x; i < n16; i += blockDim.x) {
    const uint4 v = __ldg(col4 + i);
    const unsigned int w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int q = 0; q < 4; ++q) atomicAdd(&cnt[(w[k] >> (8 * q)) & 0xffu], 1u);
  }
  for (long long i = n16 * 16 + threadIdx.x; i < n; i += blockDim.x) atomicAdd(&cnt[col[i]], 1u);
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned int best = 0u;
    int bb = 0;
    for (int b = threadIdx.x; b < 256; b += 32)
      if (cnt[b] > best) {
        best = cnt[b];
        bb = b;
      }
    for (int k = 16; k > 0; k >>= 1) {
      const unsigned int ob = __shfl_xor_sync(0xffffffffu, best, k);
      const int obb = __shfl_xor_sync(0xffffffffu, bb, k);
      if (ob > best || (ob == best && obb < bb)) {
        best = ob;
        bb = obb;
      }
    }
    if (threadIdx.x == 0) default_bin[blockIdx.x] = bb;
  }
}

// Entries of row r whose bin differs from its feature's default bin: counted
// (out == nullptr: counts[r]) or written at row_ptr[r] (f << 8 | bin, in
// feature order).  One thread per row.
__global__ void __launch_bounds__(256) k_sparse_rows(const uint8_t* __restrict__ bins_rm, long long n, int F, int Fp,
                                                    const int* __restrict__ default_bin, long long* __restrict__ counts,
                                                    const long long* __restrict__ row_ptr,
                                                    uint32_t* __restrict__ out) {
  extern __shared__ unsigned char s_def[];  // Fp bytes
  for (int f = threadIdx.x; f < Fp; f += blockDim.x) s_def[f] = f < F ? (uint8_t)default_bin[f] : 0;
  __syncthreads();
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (long long)gridDim.x * blockDim.x) {
    const uint4* row = reinterpret_cast<const uint4*>(bins_rm + r * Fp);
    long long k = out ? row_ptr[r] : 0;
    for (int c = 0; c < Fp / 16; ++c) {
      const uint4 v = __ldg(row + c);
      const unsigned int w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const int f = c * 16 + q;
        const unsigned int b = (w[q >> 2] >> (8 * (q & 3))) & 0xffu;
        if (f < F && b != s_def[f]) {
          if (out) out[k] = ((uint32_t)f << 8) | b;
          ++k;
        }
      }
    }
    if (!out) counts[r] = k;
  }
}

// Exclusive prefix sums of counts[0, n) into row_ptr[0, n] in three launches:
// block sums, a one-block scan of them, and the per-block offsets.
constexpr int kScanChunk = 1024;
__global__ void __launch_bounds__(kScanChunk) k_prefix_blocks(const long long* __restrict__ counts, long long n,
                                                              long long* __restrict__ row_ptr,
                                                              long long* __restrict__ block_sums) {
  __shared__ long long s[kScanChunk];
  const long long i = (long long)blockIdx.x * kScanChunk + threadIdx.x;
  s[threadIdx.x] = i < n ? counts[i] : 0;
  __syncthreads();
  for (int d = 1; d < kScanChunk; d <<= 1) {  // inclusive Hillis-Steele scan
    const long long v = threadIdx.x >= d ? s[threadIdx.x - d] : 0;
    __syncthreads();
    s[threadIdx.x] += v;
    __syncthreads();
  }
  if (i < n) row_ptr[i + 1] = s[threadIdx.x];
  if (threadIdx.x == kScanChunk - 1) block_sums[blockIdx.x] = s[threadIdx.x];
}
__global__ void __launch_bounds__(1024) k_prefix_sums(long long* __restrict__ block_sums, long long nb) {
  __shared__ long long s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  for (long long base = 0; base < nb; base += blockDim.x) {
    const long long i = base + threadIdx.x;
    const long long v = i < nb ? block_sums[i] : 0;
    // block-wide exclusive scan of this chunk
    __shared__ long long s[1024];
    s[threadIdx.x] = v;
    __syncthreads();
    for (int d = 1; d < (int)blockDim.x; d <<= 1) {
      const long long t = threadIdx.x >= d ? s[threadIdx.x - d] : 0;
      __syncthreads();
      s[threadIdx.x] += t;
      __syncthreads();
    }
    const long long carry = s_carry;
    if (i < nb) block_sums[i] = carry + s[threadIdx.x] - v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) s_carry = carry + s[threadIdx.x];
    __syncthreads();
  }
}
__global__ void __launch_bounds__(kScanChunk) k_prefix_add(long long n, long long* __restrict__ row_ptr,
                                                           const long long* __restrict__ block_sums) {
  const long long i = (long long)blockIdx.x * kScanChunk + threadIdx.x;
  if (i < n) row_ptr[i + 1] += block_sums[blockIdx.x];
  if (i == 0) row_ptr[0] = 0;
}

// One CTA accumulates rows [seg_b, seg_b + seg_n) of item P into its cells,
// fills in the default bins from the segment's totals and adds the cells to
// the item's work slot.  PLANES = 2: g and count (constant hessian), 3: g, h,
// count.
template <int PLANES>
__device__ void sparse_segment(const BatchItem& P, long long seg_b, long long seg_n, const uint32_t* __restrict__ entries,
                               const long long* __restrict__ row_ptr, const int* __restrict__ default_bin, int F,
                               int B, int BP, const int* __restrict__ rows0, const int* __restrict__ rows1,
                               const int2* __restrict__ pairs0, const int2* __restrict__ pairs1, int* hs,
                               unsigned int* cells, long long* s_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, n_warps = blockDim.x >> 5;
  const int* rows = P.dst_buf ? rows1 : rows0;
  const int2* pairs = P.dst_buf ? pairs1 : pairs0;
  const int plane_words = F * BP;
  const size_t words = (size_t)PLANES * plane_words;
  for (size_t c = threadIdx.x; c < words; c += blockDim.x) cells[c] = 0u;
  if (threadIdx.x < 3) s_tot[threadIdx.x] = 0;
  __syncthreads();
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(cells);
  const int bmask = BP - 1;
  long long tg = 0, th = 0;
  const long long e = seg_b + seg_n;
  for (long long c0 = seg_b + (long long)warp * 32; c0 < e; c0 += (long long)n_warps * 32) {
    const long long i = c0 + lane;
    long long pb = 0, pe = 0;
    int g = 0, h = 0;
    if (i < e) {
      const int r = __ldg(rows + i);
      const int2 pr = __ldg(pairs + i);
      g = pr.x;
      h = pr.y;
      pb = __ldg(row_ptr + r);
      pe = __ldg(row_ptr + r + 1);
      tg += g;
      th += h;
    }
    const int n_in = e - c0 < 32 ? (int)(e - c0) : 32;
    for (int u0 = 0; u0 < n_in; u0 += kSparseUnroll) {
      long long rb[kSparseUnroll], re[kSparseUnroll];
      unsigned int xg[kSparseUnroll], xh[kSparseUnroll];
#pragma unroll
      for (int u = 0; u < kSparseUnroll; ++u) {
        const int src = (u0 + u) & 31;
        rb[u] = __shfl_sync(0xffffffffu, pb, src);
        re[u] = __shfl_sync(0xffffffffu, pe, src);
        xg[u] = (unsigned int)__shfl_sync(0xffffffffu, g, src);
        xh[u] = (unsigned int)__shfl_sync(0xffffffffu, h, src);
        if (u0 + u >= n_in) re[u] = rb[u];
      }
      for (long long off = lane;; off += 32) {
        uint32_t ent[kSparseUnroll];
        bool any = false;
#pragma unroll
        for (int u = 0; u < kSparseUnroll; ++u) {
          const bool ok = rb[u] + off < re[u];
          ent[u] = ok ? __ldg(entries + rb[u] + off) : 0xffffffffu;
          any |= ok;
        }
        if (!__any_sync(0xffffffffu, any)) break;
#pragma unroll
        for (int u = 0; u < kSparseUnroll; ++u) {
          if (ent[u] == 0xffffffffu) continue;
          const int f = (int)(ent[u] >> 8), b = (int)(ent[u] & 0xffu);
          const uint32_t a = sbase + 4u * (uint32_t)(f * BP + ((b + f) & bmask));
          shared_red_add(a, xg[u]);
          if (PLANES == 3) {
            shared_red_add(a + 4u * plane_words, xh[u]);
            shared_red_add(a + 8u * plane_words, 1u);
          } else {
            shared_red_add(a + 4u * plane_words, 1u);
          }
        }
      }
    }
  }
  // segment totals: g and h over its rows, the count is seg_n
  for (int k = 16; k > 0; k >>= 1) {
    tg += __shfl_xor_sync(0xffffffffu, tg, k);
    th += __shfl_xor_sync(0xffffffffu, th, k);
  }
  if (lane == 0) {
    atomicAdd(reinterpret_cast<unsigned long long*>(&s_tot[0]), (unsigned long long)tg);
    atomicAdd(reinterpret_cast<unsigned long long*>(&s_tot[1]), (unsigned long long)th);
  }
  __syncthreads();
  // one warp per feature: lane = bin (consecutive cells of the rotated row),
  // the default bin takes the total minus the feature's listed bins
  for (int f = warp; f < F; f += n_warps) {
    const int d = default_bin[f];
#pragma unroll
    for (int p = 0; p < PLANES; ++p) {
      const long long total = p == 0 ? s_tot[0] : (PLANES == 3 && p == 1) ? s_tot[1] : seg_n;
      const int out_plane = p == 0 ? 0 : (PLANES == 3 && p == 1) ? 1 : 2;
      const unsigned int* row = cells + (size_t)p * plane_words + (size_t)f * BP;
      long long sum = 0;
      for (int b = lane; b < B; b += 32) sum += (int)row[(b + f) & bmask];
      for (int k = 16; k > 0; k >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, k);
      int* out = hs + ((long long)f * 3 + out_plane) * B;
      for (int b = lane; b < B; b += 32) {
        const int v = b == d ? (int)(total - sum) : (int)row[(b + f) & bmask];
        if (v != 0) atomicAdd(out + b, v);
      }
    }
  }
  __syncthreads();  // cells read before the next segment clears them
}

// The sparse histogram launch: one CTA per SM (clusters of one), the batch's
// built rows split over the CTAs as k_hist splits them over clusters.
template <int PLANES>
__global__ void __launch_bounds__(kSparseThreads) k_hist_sparse(
    const Batch* __restrict__ batch, const uint32_t* __restrict__ entries, const long long* __restrict__ row_ptr,
    const int* __restrict__ default_bin, int F, int B, int BP, const int* __restrict__ rows0,
    const int* __restrict__ rows1, const int2* __restrict__ pairs0, const int2* __restrict__ pairs1,
    int* __restrict__ hist, long long slot_cells, int work_base, int min_rows_per_cta, int allow_owned) {
  pdl_enter();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned int* cells = reinterpret_cast<unsigned int*>(smem_raw);
  BatchItem* s_items = reinterpret_cast<BatchItem*>(smem_raw + sparse_hist_words(PLANES, F, BP) * 4);
  long long* s_pre = reinterpret_cast<long long*>(s_items + kMaxBatch);
  int* s_asg = reinterpret_cast<int*>(s_pre + kMaxBatch + 1);  // 64 words
  long long* s_tot = reinterpret_cast<long long*>(s_asg + 64);
  const int n_items = batch->n_items;
  if (n_items == 0) return;
  {
    const int* src = reinterpret_cast<const int*>(batch->items);
    int* dst = reinterpret_cast<int*>(s_items);
    const int words = n_items * (int)(sizeof(BatchItem) / sizeof(int));
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    long long carry = 0;
    for (int base = 0; base < n_items; base += 32) {
      long long b, c = 0;
      if (base + lane < n_items) built_range(s_items[base + lane], b, c);
#pragma unroll
      for (int k = 1; k < 32; k <<= 1) {
        const long long o = __shfl_up_sync(0xffffffffu, c, k);
        if (lane >= k) c += o;
      }
      if (base + lane < n_items) s_pre[base + lane + 1] = carry + c;
      carry += __shfl_sync(0xffffffffu, c, 31);
    }
    if (lane == 0) s_pre[0] = 0;
  }
  __syncthreads();
  for_each_segment(n_items, s_items, s_pre, blockIdx.x, gridDim.x, 1, min_rows_per_cta, allow_owned, s_asg,
                   [&](const BatchItem& P, long long seg_b, long long seg_n) {
                     sparse_segment<PLANES>(P, seg_b, seg_n, entries, row_ptr, default_bin, F, B, BP, rows0, rows1,
                                            pairs0, pairs1, hist + (long long)(work_base + P.work) * slot_cells,
                                            cells, s_tot);
                   });
}

}  // namespace
}  // namespace mtb
