// Warp reductions shared by the bandwidth kernels.
#pragma once

namespace tb2 {

// Sums each of v[0 .. V) over the 32 lanes of a warp in V - 1 + 5 - log2(V)
// shuffles (V in {1, 2, 4, 8, 16, 32}): every exchange step hands half of the
// values still held to the partner lane, so after log2(V) steps each lane
// holds one index and the rest is a plain butterfly. Lane l returns the sum of
// v[l >> (5 - log2 V)] (lanes 2j and 2j + 1 both hold index j when V = 16).
// The summation order is fixed by the lane pattern alone.
template <int V>
__device__ __forceinline__ float warp_sum_multi(float (&v)[V], int lane) {
  static_assert(V == 1 || V == 2 || V == 4 || V == 8 || V == 16 || V == 32, "V must be a power of two <= 32");
  int n = V;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      n >>= 1;
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int k = 0; k < V / 2; ++k) {
        if (k < n) {
          const float send = up ? v[k] : v[k + n];
          const float keep = up ? v[k + n] : v[k];
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  return v[0];
}

// The index warp_sum_multi<V> leaves in lane l, and whether l is the first of
// the lanes holding it.
template <int V>
__device__ __forceinline__ int warp_sum_multi_index(int lane) {
  constexpr int shift = V == 1 ? 5 : V == 2 ? 4 : V == 4 ? 3 : V == 8 ? 2 : V == 16 ? 1 : 0;
  return lane >> shift;
}
template <int V>
__device__ __forceinline__ bool warp_sum_multi_leader(int lane) {
  constexpr int mask = 32 / V - 1;
  return (lane & mask) == 0;
}

}  // namespace tb2
