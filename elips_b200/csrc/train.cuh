// Device-side entry points of train.cu used by the other translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace eb {

// encode_pq (src/quant_engine/KMeans.cpp:270-285) of `n` rows [n][d] with a
// codebook [m][ksub][d/m]: codes[r][s] = the codeword nearest to the row's
// subspace s (sequential squared L2, lowest index among equal distances).
// The argmin runs on the register-tiled nearest-centroid kernel; rows go in
// chunks so the per-(row, subspace) scratch stays bounded.
// quant::detail::train_pq_codebook on device rows [n][d]: codebook [m][ksub][d/m].
void train_pq_codebook_device(int device, const float* rows, size_t n, size_t d, size_t m, size_t ksub, size_t iters,
                              float* codebook, cudaStream_t stream);

void pq_encode_device(const float* rows, size_t n, size_t d, size_t m, size_t ksub, const float* codebook,
                      uint8_t* codes, cudaStream_t stream);

}  // namespace eb
