// Materialising unpack/dequantize kernels. They exist to prove, byte for byte, that the
// register unpackers used by the decode kernels reproduce kvssd's unpack_codes and
// dequantize_tensor(q, torch.float16) (src/kvssd/quant.py:40-46, 68-73); the decode path never
// writes dequantized values to HBM.
//
// mode 0 ("row words", the K-operand path): a 32-bit word of one row is decoded into lane
//   pairs (dim k, dim k + 16/bits) exactly as the QK A fragments are built.
// mode 1 ("row pairs", the V-operand path): rows 2r and 2r+1 are interleaved lane by lane with
//   a byte permute before decoding, exactly as the PV A fragments are built.
// Both write codes (centred value + midpoint) and FP16 values in natural [row, dim] order.
#include "common.cuh"

namespace kvb {

template <int BITS>
__global__ void dequant_words_kernel(const uint8_t* __restrict__ packed,
                                     const __half* __restrict__ scales, long long rows, int d,
                                     int group, __half* __restrict__ values,
                                     uint8_t* __restrict__ codes) {
  constexpr int kPairs = LanePairs<BITS>::kPairs;  // codes per 16-bit lane
  const int words = d * BITS / 32;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * words) return;
  const long long r = i / words;
  const int wd = static_cast<int>(i - r * words);
  const int pd = d * BITS / 8, G = d / group;
  const uint32_t x = *reinterpret_cast<const uint32_t*>(packed + r * pd + wd * 4);
  const int d0 = wd * 2 * kPairs, d1 = d0 + kPairs;
  const __half2 sc = __halves2half2(scales[r * G + d0 / group], scales[r * G + d1 / group]);
  __half2 cen[kPairs], val[kPairs];
  LanePairs<BITS>::centred(x, cen);
  dequant_pairs<BITS>(x, sc, val);
  const float mid = static_cast<float>(1 << (BITS - 1));
#pragma unroll
  for (int k = 0; k < kPairs; ++k) {
    values[r * d + d0 + k] = __low2half(val[k]);
    values[r * d + d1 + k] = __high2half(val[k]);
    codes[r * d + d0 + k] = static_cast<uint8_t>(__low2float(cen[k]) + mid);
    codes[r * d + d1 + k] = static_cast<uint8_t>(__high2float(cen[k]) + mid);
  }
}

template <int BITS>
__global__ void dequant_row_pairs_kernel(const uint8_t* __restrict__ packed,
                                         const __half* __restrict__ scales, long long rows, int d,
                                         int group, __half* __restrict__ values,
                                         uint8_t* __restrict__ codes) {
  constexpr int kPairs = LanePairs<BITS>::kPairs;
  const int lanes = d * BITS / 16;  // 16-bit lanes per row
  const long long pairs = rows / 2;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= pairs * lanes) return;
  const long long rp = i / lanes;
  const int hw = static_cast<int>(i - rp * lanes);
  const int pd = d * BITS / 8, G = d / group;
  const long long r0 = 2 * rp, r1 = 2 * rp + 1;
  const uint32_t a = *reinterpret_cast<const uint32_t*>(packed + r0 * pd + (hw >> 1) * 4);
  const uint32_t b = *reinterpret_cast<const uint32_t*>(packed + r1 * pd + (hw >> 1) * 4);
  const uint32_t x = pair_lanes(a, b, hw & 1);
  const int d0 = hw * kPairs;
  const __half2 sc = __halves2half2(scales[r0 * G + d0 / group], scales[r1 * G + d0 / group]);
  __half2 cen[kPairs], val[kPairs];
  LanePairs<BITS>::centred(x, cen);
  dequant_pairs<BITS>(x, sc, val);
  const float mid = static_cast<float>(1 << (BITS - 1));
#pragma unroll
  for (int k = 0; k < kPairs; ++k) {
    values[r0 * d + d0 + k] = __low2half(val[k]);
    values[r1 * d + d0 + k] = __high2half(val[k]);
    codes[r0 * d + d0 + k] = static_cast<uint8_t>(__low2float(cen[k]) + mid);
    codes[r1 * d + d0 + k] = static_cast<uint8_t>(__high2float(cen[k]) + mid);
  }
}

using DequantKernel = void (*)(const uint8_t*, const __half*, long long, int, int, __half*,
                               uint8_t*);

DequantKernel dequant_kernel_for(int bits, int mode) {
  if (bits == 4) return mode == 0 ? dequant_words_kernel<4> : dequant_row_pairs_kernel<4>;
  if (bits == 2) return mode == 0 ? dequant_words_kernel<2> : dequant_row_pairs_kernel<2>;
  return nullptr;
}

}  // namespace kvb
