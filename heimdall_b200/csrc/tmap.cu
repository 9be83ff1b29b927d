// Host helpers: TMA tensor-map encoding through the driver entry point (resolved at run time so the
// library loads on machines without a driver), kernel attribute setup.
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_internal.h"
#include "common.cuh"
#include "tmap.h"

namespace bfb {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::mutex g_encode_mu;

static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::lock_guard<std::mutex> lk(g_encode_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return nullptr;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return g_encode;
}

int make_tmap(CUtensorMap* map, const void* base, int dtype, int rank, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  auto enc = encoder();
  if (!enc) return cuda_fail(cudaErrorNotSupported);   // no driver entry point for tensor maps
  if (reinterpret_cast<uintptr_t>(base) & 15u) return BF_ERR_ALIGNMENT;
  for (int i = 0; i < rank - 1; ++i)
    if (strides_bytes[i] & 15u) return BF_ERR_ALIGNMENT;
  CUtensorMapDataType t = dtype == BF_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                          : dtype == BF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
  CUresult r = enc(map, t, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BF_OK : cuda_fail(cudaErrorInvalidValue);   // the encoder rejected the operand
}

// K-major operand matrix [rows][K] of 16-bit elements with row stride `ld` elements, loaded as boxes of
// `box_rows` rows x (64 * atoms) columns: a 3-D map (64, rows, K/64) so that one TMA call writes
// `atoms` consecutive SW128 atom columns.
int make_tmap_kmajor(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t K, uint64_t ld,
                     uint32_t box_rows, uint32_t atoms) {
  const uint64_t dims[3] = {64, rows, (K + 63) / 64};
  const uint64_t strides[2] = {ld * 2, 128};
  const uint32_t box[3] = {64, box_rows, atoms};
  if (K % 64) return BF_ERR_UNSUPPORTED;  // atoms would straddle the end of a row
  return make_tmap(map, base, dtype, 3, dims, strides, box, true);
}

}  // namespace bfb
