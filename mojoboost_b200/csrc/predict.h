// Prediction on the device (predict.cu).
#pragma once
#include <stdint.h>

#include "model.h"

namespace mtb {

// Raw scores [n_rows][num_class] of column-major float64 rows
// (data[f * n_rows + r]) over iterations [it0, it1), on the current CUDA
// device; bit-identical to the host predictor.  Holds the rows' bins
// (n_features bytes a row) on the device for the call.
void predict_raw_device(const Model& m, const double* data, int64_t n_rows, int64_t it0, int64_t it1,
                        double* out);

}  // namespace mtb
