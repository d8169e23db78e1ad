// Element-wise int4 kernels used for exact checks and the dense drop-ins:
// unpack4 (fused_packed_moe.py:54-65) and the materialising dequant
// (`_dequant`, fused_packed_moe.py:183-189; `dequantize_weight`, quant/dequant.py:40-77).
// Neither is on the decode hot path, which never materialises weights.
#include "common.cuh"

namespace duplex {

int record_cuda(cudaError_t e);
int last_cuda_error();

__global__ void unpack4_kernel(const int32_t* __restrict__ packed, int64_t rows, int C,
                               int out_cols, int32_t* __restrict__ out) {
  const int64_t total = rows * (int64_t)out_cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / out_cols;
    const int c = (int)(i - r * out_cols);
    const uint32_t w = (uint32_t)packed[r * C + (c >> 3)];
    out[i] = (int32_t)((w >> ((c & 7) * 4)) & 0xFu) - 8;
  }
}

template <typename S, typename O>
__global__ void dequant_kernel(const int32_t* __restrict__ packed, const S* __restrict__ scale,
                               const int32_t* __restrict__ zeros, int64_t rows, int K, int group,
                               int G, int GZ, O* __restrict__ out) {
  const int64_t total = rows * (int64_t)K;
  const int C = K >> 3;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K;
    const int c = (int)(i - r * K);
    const uint32_t w = (uint32_t)packed[r * C + (c >> 3)];
    const int nib = (int)((w >> ((c & 7) * 4)) & 0xFu);
    const int grp = c / group;
    int z = 8;
    if (zeros) z = (int)(((uint32_t)zeros[r * GZ + (grp >> 3)] >> ((grp & 7) * 4)) & 0xFu);
    const float s = to_f32<S>(scale[r * G + grp]);
    // (nib - z) * s is exact in fp32 for 16-bit scales; for fp32 scales it is the
    // single fp32 rounding the reference performs.  One rounding into O follows.
    out[i] = from_f32<O>((float)(nib - z) * s);
  }
}

template <typename S>
static int dequant_out(const int32_t* packed, const S* scale, const int32_t* zeros, int64_t rows,
                       int K, int group, void* out, int out_dtype, cudaStream_t st) {
  const int G = (K + group - 1) / group, GZ = (G + 7) / 8;
  const int64_t total = rows * (int64_t)K;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  if (out_dtype == DUPLEX_DTYPE_F16)
    dequant_kernel<S, __half><<<blocks, 256, 0, st>>>(packed, scale, zeros, rows, K, group, G, GZ,
                                                      reinterpret_cast<__half*>(out));
  else if (out_dtype == DUPLEX_DTYPE_BF16)
    dequant_kernel<S, __nv_bfloat16><<<blocks, 256, 0, st>>>(
        packed, scale, zeros, rows, K, group, G, GZ, reinterpret_cast<__nv_bfloat16*>(out));
  else if (out_dtype == DUPLEX_DTYPE_F32)
    dequant_kernel<S, float><<<blocks, 256, 0, st>>>(packed, scale, zeros, rows, K, group, G, GZ,
                                                     reinterpret_cast<float*>(out));
  else
    return DUPLEX_ERR_DTYPE;
  return record_cuda(cudaGetLastError());
}

}  // namespace duplex

using namespace duplex;

extern "C" int duplex_version(void) { return 100; }

extern "C" const char* duplex_error_string(int status) {
  switch (status) {
    case DUPLEX_OK: return "ok";
    case DUPLEX_ERR_ARG: return "invalid argument (size, null pointer or combination)";
    case DUPLEX_ERR_ALIGN: return "pointer or stride is not 16-byte aligned";
    case DUPLEX_ERR_DTYPE: return "unsupported dtype";
    case DUPLEX_ERR_WORKSPACE: return "workspace too small";
    case DUPLEX_ERR_CUDA: return "CUDA runtime error";
    case DUPLEX_ERR_UNSUPPORTED: return "shape not supported by the kernels";
    case DUPLEX_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the no-allocation entry point's static array";
    default: return "unknown status";
  }
}

extern "C" int duplex_last_cuda_error(void) { return last_cuda_error(); }

extern "C" int duplex_unpack4(const int32_t* packed, int64_t rows, int32_t C, int32_t out_cols,
                              int32_t* out, void* stream) {
  if (!packed || !out || rows < 0 || C < 1 || out_cols < 0 || out_cols > 8 * C)
    return DUPLEX_ERR_ARG;
  const int64_t total = rows * (int64_t)out_cols;
  if (total == 0) return DUPLEX_OK;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  unpack4_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(packed, rows, C, out_cols, out);
  return record_cuda(cudaGetLastError());
}

extern "C" int duplex_dequant(const int32_t* packed, const void* scale, int scale_dtype,
                              const int32_t* zeros, int64_t rows, int32_t K, int32_t group,
                              void* out, int out_dtype, void* stream) {
  if (!packed || !scale || !out || rows < 0 || K < 8 || (K & 7) || group < 1) return DUPLEX_ERR_ARG;
  if (rows == 0) return DUPLEX_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (scale_dtype == DUPLEX_DTYPE_F16)
    return dequant_out(packed, reinterpret_cast<const __half*>(scale), zeros, rows, K, group, out,
                       out_dtype, st);
  if (scale_dtype == DUPLEX_DTYPE_BF16)
    return dequant_out(packed, reinterpret_cast<const __nv_bfloat16*>(scale), zeros, rows, K, group,
                       out, out_dtype, st);
  if (scale_dtype == DUPLEX_DTYPE_F32)
    return dequant_out(packed, reinterpret_cast<const float*>(scale), zeros, rows, K, group, out,
                       out_dtype, st);
  return DUPLEX_ERR_DTYPE;
}
