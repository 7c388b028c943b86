// ltx25-adaln.h -- the trunk's adaLN chains on the host: the timestep
// sinusoid and the three-linear MLP that turns one noise level into a
// block's modulation driver (Ltx25Dit::adaln_, src/ltx25-dit.cc:51-160).
// The reference runs them as host GEMVs over bf16 weights with f64 sums,
// once per denoise level and step, before the block loop; so does this,
// split over host threads by output row, each row summed in a fixed order
// (sixteen interleaved partial sums; AVX2 + FMA where the host has it,
// LTX25_HOST_SIMD=0 forces the scalar form, which gives the same bits).
#pragma once

#include <cstdint>
#include <vector>

namespace ltx25 {

struct AdaLNChain {
  int dim = 0, out_dim = 0;
  // bf16 bits, [out][in]: emb.timestep_embedder.linear_1 (256 -> dim),
  // linear_2 (dim -> dim), and the root `linear` (dim -> out_dim)
  std::vector<uint16_t> w1, b1, w2, b2, w3, b3;
};

// The 256-channel sinusoid of `t` (max period 10000, downscale shift 0,
// flip_sin_to_cos: [cos | sin]), src/ltx25-dit.cc:109-132.
void timestep_sinusoid(double t, int channels, float* out);

// out [out_dim] = linear(silu(h2)), embedded [dim] = h2 = linear_2(silu(
// linear_1(sinusoid(t)))) (may be null); `threads` <= 0: the host's count.
void adaln_run(const AdaLNChain& c, double t, float* out, float* embedded, int threads);

// `count` chains at once (a denoise step's chains, each at its own
// timestep): each stage's rows over all chains are split evenly over the
// host threads, the stages one after another.  Every row is summed exactly
// as adaln_run sums it, so the results are the same bits.  embedded (or any
// of its entries) may be null.
void adaln_run_many(const AdaLNChain* const* chains, const double* t, float* const* out,
                    float* const* embedded, int count, int threads);

}  // namespace ltx25
