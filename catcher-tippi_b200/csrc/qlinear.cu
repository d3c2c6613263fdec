// C++ host layer: device contexts, weight binding, shape validation and
// kernel dispatch for the quantized linear.  See qlinear.hpp.
#include "qlinear.hpp"

#include <cudaTypedefs.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "common.cuh"
#include "qops.hpp"

namespace nemotron_cuda {

namespace {

std::string fmt_shape_error(const char* prefix, const std::string& msg) {
  return std::string(prefix) + msg;
}

thread_local int t_pdl = -1;  // -1: the default

}  // namespace

bool pdl_default() { return true; }

bool pdl_enabled() { return t_pdl >= 0 ? t_pdl != 0 : pdl_default(); }

PdlScope::PdlScope(bool on) : prev_(t_pdl) { t_pdl = on ? 1 : 0; }
PdlScope::~PdlScope() { t_pdl = prev_; }

namespace {

void validate_group(int group) {
  if (group != 32 && group != 64 && group != 128) {
    std::ostringstream os;
    os << "group size " << group << " is not supported; supported group sizes are 32, 64 and 128";
    throw_invalid(os.str());
  }
}

void validate_dtype(cq_dtype dtype) {
  if (dtype != CQ_F16 && dtype != CQ_BF16 && dtype != CQ_F32)
    throw_invalid("unknown dtype " + std::to_string(dtype));
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr int kMaxInputDims = 8192;

}  // namespace

[[noreturn]] void throw_invalid(const std::string& msg) { throw Error(CQ_INVALID_ARGUMENT, msg); }

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear a sticky launch error so later calls report their own
    throw Error(CQ_RUNTIME_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

size_t dtype_size(cq_dtype dtype) { return dtype == CQ_F32 ? 4 : 2; }

DeviceGuard::DeviceGuard(int device) {
  check_cuda(cudaGetDevice(&prev_), "cudaGetDevice");
  if (prev_ != device) check_cuda(cudaSetDevice(device), "cudaSetDevice");
}

DeviceGuard::~DeviceGuard() {
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur != prev_ && prev_ >= 0) cudaSetDevice(prev_);
}

DeviceContext& device_context(int device) {
  static std::mutex mu;
  static std::vector<std::unique_ptr<DeviceContext>> contexts;
  std::lock_guard<std::mutex> lock(mu);
  int count = 0;
  check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count)
    throw_invalid("device " + std::to_string(device) + " does not exist (" +
                  std::to_string(count) + " visible)");
  if (contexts.size() < static_cast<size_t>(count)) contexts.resize(count);
  if (!contexts[device]) {
    DeviceGuard guard(device);
    auto ctx = std::make_unique<DeviceContext>();
    ctx->device = device;
    int major = 0, minor = 0;
    check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), "attr");
    check_cuda(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device), "attr");
    if (major != 10)
      throw Error(CQ_RUNTIME_ERROR, "device " + std::to_string(device) + " is sm_" +
                                        std::to_string(major) + std::to_string(minor) +
                                        "; this library is built for sm_100a only");
    check_cuda(cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device),
               "attr");
    check_cuda(cudaMalloc(&ctx->status, sizeof(int)), "cudaMalloc(status)");
    check_cuda(cudaMemset(ctx->status, 0, sizeof(int)), "cudaMemset(status)");
    contexts[device] = std::move(ctx);
  }
  return *contexts[device];
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qres{};
    check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres),
               "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (fn == nullptr || qres != cudaDriverEntryPointSuccess)
      throw Error(CQ_RUNTIME_ERROR, "cuTensorMapEncodeTiled is unavailable");
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return encode;
}

CUtensorMap encode_map(CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                       const cuuint64_t* strides, const cuuint32_t* box,
                       CUtensorMapSwizzle swizzle) {
  CUtensorMap map{};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = tensor_map_encoder()(&map, dt, rank, const_cast<void*>(base), dims, strides, box,
                                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(CQ_RUNTIME_ERROR, "cuTensorMapEncodeTiled failed with " + std::to_string(r));
  return map;
}

}  // namespace

CUtensorMap make_map_2d(const void* base, int elem_bytes, int rows, int cols, int ld,
                        int box_rows, int box_cols, CUtensorMapSwizzle swizzle) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * elem_bytes};  // bytes per row
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const CUtensorMapDataType dt =
      elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode_map(dt, 2, base, dims, strides, box, swizzle);
}

cq::GemmActMaps make_act_maps(const void* base, int rows, int K, int ld, int tn) {
  cq::GemmActMaps m{};
  m.tn = tn;
  m.tile = make_map_2d(base, 2, rows, K, ld, tn, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  const int full = K / 64;
  if (full >= 2) {
    // {64 k, rows, k-tile}: element (k, r, t) at r * ld + 64 t + k; only the
    // full k-tiles, so no copy reaches past a row's K elements
    const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(full)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2, 128};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(tn), 2};
    m.pair = encode_map(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    m.pair_tiles = full;
  } else {
    m.pair = m.tile;
    m.pair_tiles = 0;
  }
  return m;
}

// ------------------------------------------------------------------ layer

QuantizedLinear::QuantizedLinear(int N, int K, int group, cq_dtype dtype, int device)
    : N_(N), K_(K), group_(group), dtype_(dtype), device_(device) {}

QuantizedLinear::~QuantizedLinear() {
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device_);
  cudaFree(q_);
  cudaFree(scales_);
  cudaFree(biases_);
  cudaFree(bias_);
  cudaFree(host_scratch_);
  cudaFree(ws_);
  cudaFree(sb_tiles_);
  if (prev >= 0) cudaSetDevice(prev);
}

void QuantizedLinear::allocate(bool with_bias) {
  const size_t groups = static_cast<size_t>(N_) * (K_ / group_);
  check_cuda(cudaMalloc(&q_, static_cast<size_t>(N_) * K_), "cudaMalloc(qweight)");
  check_cuda(cudaMalloc(&scales_, groups * dtype_size(dtype_)), "cudaMalloc(scales)");
  check_cuda(cudaMalloc(&biases_, groups * dtype_size(dtype_)), "cudaMalloc(biases)");
  if (with_bias) check_cuda(cudaMalloc(&bias_, N_ * dtype_size(dtype_)), "cudaMalloc(bias)");
}

void QuantizedLinear::finalize() {
  if (dtype_ == CQ_F32) return;  // the f32 path uses the CUDA-core kernel
  // K1 holds at most 16 sub-blocks of 64 per CTA and splits K over a
  // portable cluster of at most 8 CTAs.
  if (K_ > kMaxInputDims)
    throw_invalid("input_dims " + std::to_string(K_) + " exceeds the supported maximum " +
                  std::to_string(kMaxInputDims));
  DeviceContext& ctx = device_context(device_);
  plan_ = cq::plan_gemv(N_, K_, ctx.num_sms);
  wmap_ = make_map_2d(q_, 1, N_, K_, K_, 16 * plan_.rt, 64, CU_TENSOR_MAP_SWIZZLE_NONE);
  for (int i = 0; i < 3; ++i)
    wmap_rt_[i] = make_map_2d(q_, 1, N_, K_, K_, 16 << i, 64, CU_TENSOR_MAP_SWIZZLE_NONE);
  // K2 copies two 64-wide k-tiles of packed weights at a time
  gemm_ok_ = K_ >= 128 && check_f16_range();
  if (gemm_ok_) {
    qmap_gemm_ = make_map_2d(q_, 1, N_, K_, K_, cq::kGemmBN, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    check_cuda(cudaMalloc(&sb_tiles_, cq::sb_tiles_bytes(N_, K_, group_)), "cudaMalloc(sb tiles)");
    check_cuda(cq::build_sb_tiles(dtype_, scales_, biases_, N_, K_, group_, sb_tiles_, nullptr),
               "build sb tiles");
    check_cuda(cudaDeviceSynchronize(), "build sb tiles");
  }
}

// K2 dequantises to f16.  f16 layers are exact by construction; a bf16 layer
// qualifies when every nonzero scale is an f16 normal number and every
// dequantised weight (|s| * 255 + |b|) stays below the f16 maximum.
bool QuantizedLinear::check_f16_range() const {
  if (dtype_ == CQ_F16) return true;
  if (dtype_ != CQ_BF16) return false;
  const size_t groups = static_cast<size_t>(N_) * (K_ / group_);
  std::vector<uint16_t> s(groups), b(groups);
  check_cuda(cudaMemcpy(s.data(), scales_, groups * 2, cudaMemcpyDeviceToHost), "read scales");
  check_cuda(cudaMemcpy(b.data(), biases_, groups * 2, cudaMemcpyDeviceToHost), "read biases");
  auto widen = [](uint16_t v) {
    uint32_t u = static_cast<uint32_t>(v) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  };
  for (size_t i = 0; i < groups; ++i) {
    const float sv = std::fabs(widen(s[i])), bv = std::fabs(widen(b[i]));
    if (!(sv == 0.0f || (sv >= 6.103515625e-05f && sv <= 65504.0f))) return false;
    if (!(sv * 255.0f + bv <= 65504.0f)) return false;  // also rejects NaN/inf
  }
  return true;
}

void QuantizedLinear::reserve(int max_rows) {
  if (max_rows < 0) throw_invalid("reserve: negative row count");
  if (dtype_ != CQ_BF16 || !gemm_ok_ || max_rows < cq::kGemmMinRows) return;
  std::lock_guard<std::mutex> lock(ws_mu_);
  if (max_rows <= ws_rows_) return;
  DeviceGuard guard(device_);
  const size_t xbytes = align_up(static_cast<size_t>(max_rows) * K_ * 2, 256);
  const size_t need = xbytes + static_cast<size_t>(max_rows) * sizeof(float);
  void* p = nullptr;
  check_cuda(cudaMalloc(&p, need), "cudaMalloc(gemm workspace)");
  cudaFree(ws_);
  ws_ = p;
  ws_bytes_ = need;
  ws_rows_ = max_rows;
  amap_ptr_ = nullptr;  // the cached map may point into the old workspace
}

void QuantizedLinear::forward_gemm(const void* x, int ldx, int rows, void* y, int ldy, int act,
                                   cudaStream_t stream) {
  DeviceContext& ctx = device_context(device_);
  const void* a_ptr = x;
  int a_ld = ldx;
  const float* row_scale = nullptr;
  if (dtype_ == CQ_BF16) {
    reserve(rows);
    const size_t xbytes = align_up(static_cast<size_t>(ws_rows_) * K_ * 2, 256);
    float* rs = reinterpret_cast<float*>(static_cast<char*>(ws_) + xbytes);
    check_cuda(cq::launch_gemm_prepass(x, ldx, rows, K_, ws_, K_, rs, stream, pdl_enabled()),
               "qgemm prepass");
    a_ptr = ws_;
    a_ld = K_;
    row_scale = rs;
  }
  if (a_ptr != amap_ptr_ || a_ld != amap_ld_ || rows != amap_rows_) {
    amap_ = make_act_maps(a_ptr, rows, K_, a_ld, cq::gemm_tile_tokens(rows, N_, K_, ctx.num_sms));
    amap_ptr_ = a_ptr;
    amap_ld_ = a_ld;
    amap_rows_ = rows;
  }
  cq::GemmArgs g{};
  g.row_scale = row_scale;
  g.sb_tiles = sb_tiles_;
  g.bias = bias_;
  g.y = y;
  g.status = ctx.status;
  g.M = rows;
  g.N = N_;
  g.K = K_;
  g.ldy = ldy;
  g.act = act;
  g.tn = amap_.tn;
  g.splits = cq::gemm_splits(rows, N_, K_, ctx.num_sms, g.tn);
  g.pair_tiles = amap_.pair_tiles;
  check_cuda(cq::launch_gemm(dtype_, group_, amap_, qmap_gemm_, g, stream, pdl_enabled()), "qgemm");
}

bool QuantizedLinear::gemm_for(int rows) const {
  return dtype_ == CQ_BF16 && gemm_ok_ && rows >= cq::kGemmMinRows;
}

void QuantizedLinear::forward_prescaled(const void* x16, const float* row_scale, int rows, void* y,
                                        int ldy, int act, cudaStream_t stream) {
  if (!gemm_for(rows)) throw_invalid("prescaled activations feed only the bf16 tensor-core GEMM");
  if (x16 == nullptr || row_scale == nullptr || y == nullptr)
    throw_invalid("input, row scales and output must not be null");
  if (ldy < N_) throw_invalid("output leading dimension is smaller than the layer");
  if ((reinterpret_cast<uintptr_t>(x16) & 15) != 0 || (K_ % 8) != 0)
    throw_invalid("prescaled rows must be 16-byte aligned");
  if (act != CQ_ACT_NONE && act != CQ_ACT_SILU && act != CQ_ACT_RELU)
    throw_invalid("unknown activation " + std::to_string(act));
  DeviceContext& ctx = device_context(device_);
  DeviceGuard guard(device_);
  if (x16 != amap_pre_ptr_ || rows != amap_pre_rows_) {
    amap_pre_ = make_act_maps(x16, rows, K_, K_, cq::gemm_tile_tokens(rows, N_, K_, ctx.num_sms));
    amap_pre_ptr_ = x16;
    amap_pre_rows_ = rows;
  }
  cq::GemmArgs g{};
  g.row_scale = row_scale;
  g.sb_tiles = sb_tiles_;
  g.bias = bias_;
  g.y = y;
  g.status = ctx.status;
  g.M = rows;
  g.N = N_;
  g.K = K_;
  g.ldy = ldy;
  g.act = act;
  g.tn = amap_pre_.tn;
  g.splits = cq::gemm_splits(rows, N_, K_, ctx.num_sms, g.tn);
  g.pair_tiles = amap_pre_.pair_tiles;
  check_cuda(cq::launch_gemm(dtype_, group_, amap_pre_, qmap_gemm_, g, stream, pdl_enabled()),
             "qgemm");
}

void QuantizedLinear::prescale(const void* x, int ldx, int rows, void* x16, float* row_scale,
                               cudaStream_t stream) {
  if (!gemm_for(rows))
    throw_invalid("the tensor-core activation format applies to bf16 layers at >= " +
                  std::to_string(cq::kGemmMinRows) + " rows");
  if (x == nullptr || x16 == nullptr || row_scale == nullptr)
    throw_invalid("input, prescaled output and row scales must not be null");
  if (ldx < K_) throw_invalid("input leading dimension is smaller than the layer");
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (ldx % 8) != 0 ||
      (reinterpret_cast<uintptr_t>(x16) & 15) != 0 || (K_ % 8) != 0)
    throw_invalid("input and prescaled rows must be 16-byte aligned");
  DeviceGuard guard(device_);
  check_cuda(cq::launch_gemm_prepass(x, ldx, rows, K_, x16, K_, row_scale, stream, pdl_enabled()),
             "qgemm prepass");
}

size_t QuantizedLinear::scratch_bytes_for(int rows) const {
  if (dtype_ != CQ_BF16 || !gemm_ok_ || rows < cq::kGemmMinRows) return 0;
  return align_up(static_cast<size_t>(rows) * K_ * 2, 256) + static_cast<size_t>(rows) * 4;
}

void QuantizedLinear::forward_array_in_scratch(const void* x, int ldx, int rows, void* y, int ldy,
                                               int act, cudaStream_t stream, void* scratch,
                                               size_t scratch_bytes) {
  const size_t need = rows > 0 ? scratch_bytes_for(rows) : 0;
  if (need == 0) {
    // the GEMV, the f16 GEMM and the f32 path stage nothing
    forward_array(x, ldx, rows, y, ldy, act, stream);
    return;
  }
  if (need > scratch_bytes)
    throw_invalid("rows x input_dims = " + std::to_string(rows) + "x" + std::to_string(K_) +
                  " needs " + std::to_string(need) + " bytes of scratch; the no-allocation limit is " +
                  std::to_string(scratch_bytes) + " bytes");
  if (x == nullptr || y == nullptr || scratch == nullptr)
    throw_invalid("input, output and scratch must not be null");
  if (ldx < K_ || ldy < N_)
    throw_invalid("leading dimensions (" + std::to_string(ldx) + ", " + std::to_string(ldy) +
                  ") are smaller than the layer (" + std::to_string(K_) + ", " +
                  std::to_string(N_) + ")");
  if (act != CQ_ACT_NONE && act != CQ_ACT_SILU && act != CQ_ACT_RELU)
    throw_invalid("unknown activation " + std::to_string(act));
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (ldx % 8) != 0)
    throw_invalid("input rows must be 16-byte aligned (x % 16 == 0 and ldx % 8 == 0)");
  DeviceContext& ctx = device_context(device_);
  DeviceGuard guard(device_);
  const size_t xbytes = align_up(static_cast<size_t>(rows) * K_ * 2, 256);
  float* rs = reinterpret_cast<float*>(static_cast<char*>(scratch) + xbytes);
  check_cuda(cq::launch_gemm_prepass(x, ldx, rows, K_, scratch, K_, rs, stream, pdl_enabled()),
             "qgemm prepass");
  if (scratch != amap_scratch_ptr_ || rows != amap_scratch_rows_) {
    amap_scratch_ = make_act_maps(scratch, rows, K_, K_, cq::gemm_tile_tokens(rows, N_, K_, ctx.num_sms));
    amap_scratch_ptr_ = scratch;
    amap_scratch_rows_ = rows;
  }
  cq::GemmArgs g{};
  g.row_scale = rs;
  g.sb_tiles = sb_tiles_;
  g.bias = bias_;
  g.y = y;
  g.status = ctx.status;
  g.M = rows;
  g.N = N_;
  g.K = K_;
  g.ldy = ldy;
  g.act = act;
  g.tn = amap_scratch_.tn;
  g.splits = cq::gemm_splits(rows, N_, K_, ctx.num_sms, g.tn);
  g.pair_tiles = amap_scratch_.pair_tiles;
  check_cuda(cq::launch_gemm(dtype_, group_, amap_scratch_, qmap_gemm_, g, stream, pdl_enabled()),
             "qgemm");
}

std::unique_ptr<QuantizedLinear> QuantizedLinear::from_packed(const uint32_t* qweight,
                                                              const void* scales,
                                                              const void* biases, const void* bias,
                                                              int output_dims, int input_dims,
                                                              int group, cq_dtype dtype,
                                                              int device) {
  if (qweight == nullptr || scales == nullptr || biases == nullptr)
    throw_invalid("qweight, scales and biases must not be null");
  validate_dtype(dtype);
  if (output_dims <= 0 || input_dims <= 0)
    throw_invalid("invalid model shape: linear dimensions must be positive, got " +
                  std::to_string(output_dims) + "x" + std::to_string(input_dims));
  validate_group(group);
  if (input_dims % group != 0)
    throw_invalid("invalid model shape: linear input dimension " + std::to_string(input_dims) +
                  " is incompatible with group size " + std::to_string(group));
  device_context(device);
  DeviceGuard guard(device);
  std::unique_ptr<QuantizedLinear> L(
      new QuantizedLinear(output_dims, input_dims, group, dtype, device));
  L->allocate(bias != nullptr);
  const size_t groups = static_cast<size_t>(output_dims) * (input_dims / group);
  // cudaMemcpyDefault: the source arrays may live in host or device memory.
  check_cuda(cudaMemcpy(L->q_, qweight, static_cast<size_t>(output_dims) * input_dims,
                        cudaMemcpyDefault),
             "copy qweight");
  check_cuda(cudaMemcpy(L->scales_, scales, groups * dtype_size(dtype), cudaMemcpyDefault),
             "copy scales");
  check_cuda(cudaMemcpy(L->biases_, biases, groups * dtype_size(dtype), cudaMemcpyDefault),
             "copy biases");
  if (bias != nullptr)
    check_cuda(cudaMemcpy(L->bias_, bias, output_dims * dtype_size(dtype), cudaMemcpyDefault),
               "copy bias");
  check_cuda(cudaDeviceSynchronize(), "copy weights");
  L->finalize();
  return L;
}

std::unique_ptr<QuantizedLinear> QuantizedLinear::from_f32(const float* weight, size_t weight_len,
                                                           int output_dims, int input_dims,
                                                           const float* bias, size_t bias_len,
                                                           int group, cq_dtype dtype, int device) {
  // validate_linear_shapes (crates/nemotron-mlx/src/model/layers.rs:510-530)
  const std::string dims = std::to_string(output_dims) + "x" + std::to_string(input_dims);
  if (output_dims < 0 || input_dims < 0 ||
      static_cast<size_t>(output_dims) * static_cast<size_t>(input_dims) != weight_len ||
      bias_len != static_cast<size_t>(output_dims))
    throw_invalid("invalid model shape: linear weight/bias mismatch for " + dims);
  if (group <= 0 || input_dims % group != 0)
    throw_invalid("invalid model shape: linear input dimension " + std::to_string(input_dims) +
                  " is incompatible with group size " + std::to_string(group));
  if ((weight == nullptr && weight_len > 0) || (bias == nullptr && bias_len > 0))
    throw_invalid("weight and bias must not be null");
  validate_dtype(dtype);
  validate_group(group);
  if (output_dims == 0 || input_dims == 0)
    throw_invalid("invalid model shape: linear dimensions must be positive, got " + dims);
  device_context(device);
  DeviceGuard guard(device);
  std::unique_ptr<QuantizedLinear> L(
      new QuantizedLinear(output_dims, input_dims, group, dtype, device));
  L->allocate(true);
  float* dw = nullptr;
  float* db = nullptr;
  check_cuda(cudaMalloc(&dw, weight_len * sizeof(float)), "cudaMalloc(weight)");
  check_cuda(cudaMalloc(&db, bias_len * sizeof(float)), "cudaMalloc(bias f32)");
  cudaError_t e = cudaMemcpy(dw, weight, weight_len * sizeof(float), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(db, bias, bias_len * sizeof(float), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cq::launch_quantize(dtype, dw, output_dims, input_dims, group, dtype != CQ_F32, L->q_,
                            L->scales_, L->biases_, nullptr);
  if (e == cudaSuccess) e = cq::launch_f32_to_t(dtype, db, bias_len, L->bias_, nullptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(dw);
  cudaFree(db);
  check_cuda(e, "quantize weight");
  L->finalize();
  return L;
}

std::unique_ptr<QuantizedLinear> QuantizedLinear::concat(
    const std::vector<const QuantizedLinear*>& parts) {
  if (parts.empty()) throw_invalid("concat needs at least one layer");
  for (const auto* p : parts)
    if (p == nullptr) throw_invalid("concat: null layer");
  const QuantizedLinear& f = *parts[0];
  int total_n = 0;
  bool any_bias = false;
  for (const auto* p : parts) {
    if (p->K_ != f.K_ || p->group_ != f.group_ || p->dtype_ != f.dtype_ || p->device_ != f.device_)
      throw_invalid("concat: layers differ in input_dims, group size, dtype or device");
    total_n += p->N_;
    any_bias = any_bias || p->bias_ != nullptr;
  }
  DeviceGuard guard(f.device_);
  std::unique_ptr<QuantizedLinear> L(
      new QuantizedLinear(total_n, f.K_, f.group_, f.dtype_, f.device_));
  L->allocate(any_bias);
  const size_t es = dtype_size(f.dtype_);
  const size_t gpr = f.K_ / f.group_;
  size_t row = 0;
  for (const auto* p : parts) {
    check_cuda(cudaMemcpy(L->q_ + row * f.K_, p->q_, static_cast<size_t>(p->N_) * f.K_,
                          cudaMemcpyDeviceToDevice),
               "concat qweight");
    check_cuda(cudaMemcpy(static_cast<char*>(L->scales_) + row * gpr * es, p->scales_,
                          p->N_ * gpr * es, cudaMemcpyDeviceToDevice),
               "concat scales");
    check_cuda(cudaMemcpy(static_cast<char*>(L->biases_) + row * gpr * es, p->biases_,
                          p->N_ * gpr * es, cudaMemcpyDeviceToDevice),
               "concat biases");
    if (any_bias) {
      char* dst = static_cast<char*>(L->bias_) + row * es;
      if (p->bias_ != nullptr)
        check_cuda(cudaMemcpy(dst, p->bias_, p->N_ * es, cudaMemcpyDeviceToDevice), "concat bias");
      else
        check_cuda(cudaMemset(dst, 0, p->N_ * es), "concat zero bias");
    }
    row += p->N_;
  }
  L->finalize();
  return L;
}

void QuantizedLinear::forward_array(const void* x, int ldx, int rows, void* y, int ldy, int act,
                                    cudaStream_t stream) const {
  if (rows < 0) throw_invalid("invalid model shape: negative row count");
  if (rows == 0) return;
  if (x == nullptr || y == nullptr) throw_invalid("input and output must not be null");
  if (ldx < K_ || ldy < N_)
    throw_invalid("leading dimensions (" + std::to_string(ldx) + ", " + std::to_string(ldy) +
                  ") are smaller than the layer (" + std::to_string(K_) + ", " +
                  std::to_string(N_) + ")");
  if (act != CQ_ACT_NONE && act != CQ_ACT_SILU && act != CQ_ACT_RELU)
    throw_invalid("unknown activation " + std::to_string(act));
  DeviceContext& ctx = device_context(device_);
  DeviceGuard guard(device_);
  if (dtype_ == CQ_F32) {
    if (ldx != K_ || ldy != N_ || act != CQ_ACT_NONE)
      throw_invalid("the f32 path takes contiguous rows and no fused activation");
    check_cuda(cq::launch_qmatmul_f32(static_cast<const float*>(x), rows, K_, q_,
                                      static_cast<const float*>(scales_),
                                      static_cast<const float*>(biases_), N_, group_,
                                      static_cast<float*>(y), stream),
               "qmatmul_f32");
    return;
  }
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (ldx % 8) != 0)
    throw_invalid("input rows must be 16-byte aligned (x % 16 == 0 and ldx % 8 == 0)");
  if (rows >= cq::kGemmMinRows && gemm_ok_) {
    const_cast<QuantizedLinear*>(this)->forward_gemm(x, ldx, rows, y, ldy, act, stream);
    return;
  }
  cq::GemvArgs a{};
  a.x = x;
  a.scales = scales_;
  a.biases = biases_;
  a.bias = bias_;
  a.y = y;
  a.status = ctx.status;
  a.M = rows;
  a.N = N_;
  a.K = K_;
  a.ldx = ldx;
  a.ldy = ldy;
  a.sb_per_cta = plan_.sb_per_cta;
  a.act = act;
  const cq::GemvPlan plan = cq::plan_gemv_rows(plan_, N_, rows);
  const CUtensorMap& wmap = plan.rt == plan_.rt ? wmap_ : wmap_rt_[plan.rt == 1 ? 0 : plan.rt == 2 ? 1 : 2];
  check_cuda(cq::launch_gemv(dtype_, group_, plan, wmap, a, stream, pdl_enabled()), "qgemv");
}

bool QuantizedLinear::rnnt_epilogue_fits(int rows) const {
  return (dtype_ == CQ_F16 || dtype_ == CQ_BF16) && rows >= 1 && rows < cq::kGemmMinRows &&
         cq::plan_gemv_rows(plan_, N_, rows).ksplit == 1 && K_ % 8 == 0;
}

void QuantizedLinear::forward_rnnt(const void* x, int ldx, int rows, void* y, int ldy, int mode,
                                   const cq::RnntEpilogue& epi, cudaStream_t stream) const {
  if (!rnnt_epilogue_fits(rows)) throw_invalid("the RNNT epilogues run on the one-CTA GEMV");
  if (x == nullptr || y == nullptr) throw_invalid("input and output must not be null");
  if (ldx < K_ || ldy < N_) throw_invalid("leading dimensions are smaller than the layer");
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (ldx % 8) != 0)
    throw_invalid("input rows must be 16-byte aligned (x % 16 == 0 and ldx % 8 == 0)");
  DeviceContext& ctx = device_context(device_);
  DeviceGuard guard(device_);
  const cq::GemvPlan plan = cq::plan_gemv_rows(plan_, N_, rows);
  cq::GemvMaps maps;
  maps.m[0] = plan.rt == plan_.rt ? wmap_ : wmap_rt_[plan.rt == 1 ? 0 : plan.rt == 2 ? 1 : 2];
  cq::GemvGroup g{};
  g.count = 1;
  cq::GemvArgs& a = g.a[0];
  a.x = x;
  a.scales = scales_;
  a.biases = biases_;
  a.bias = bias_;
  a.y = y;
  a.status = ctx.status;
  a.M = rows;
  a.N = N_;
  a.K = K_;
  a.ldx = ldx;
  a.ldy = ldy;
  a.sb_per_cta = plan_.sb_per_cta;
  a.act = CQ_ACT_NONE;
  a.mode = mode;
  check_cuda(cq::launch_gemv_group(dtype_, group_, plan, maps, g, stream, pdl_enabled(), &epi),
             "qgemv (RNNT epilogue)");
}

void QuantizedLinear::forward_group(const GroupCall* calls, int count, int rows, int act,
                                    cudaStream_t stream) {
  if (calls == nullptr || count < 1 || count > cq::kGemvMaxGroup)
    throw_invalid("a linear group holds 1.." + std::to_string(cq::kGemvMaxGroup) + " calls");
  const QuantizedLinear& L0 = *calls[0].layer;
  if (rows < 1 || rows >= cq::kGemmMinRows)
    throw_invalid("grouped linears take 1.." + std::to_string(cq::kGemmMinRows - 1) + " rows");
  if (L0.dtype_ != CQ_F16 && L0.dtype_ != CQ_BF16) throw_invalid("grouped linears run f16 or bf16");
  if (act != CQ_ACT_NONE && act != CQ_ACT_SILU && act != CQ_ACT_RELU)
    throw_invalid("unknown activation " + std::to_string(act));
  DeviceContext& ctx = device_context(L0.device_);
  DeviceGuard guard(L0.device_);
  const cq::GemvPlan plan = cq::plan_gemv_rows(L0.plan_, L0.N_, rows);
  cq::GemvMaps maps;
  cq::GemvGroup g{};
  g.count = count;
  for (int i = 0; i < count; ++i) {
    const GroupCall& c = calls[i];
    if (c.layer == nullptr || c.x == nullptr || c.y == nullptr)
      throw_invalid("grouped linear calls need a layer, an input and an output");
    const QuantizedLinear& L = *c.layer;
    if (L.N_ != L0.N_ || L.K_ != L0.K_ || L.group_ != L0.group_ || L.dtype_ != L0.dtype_ ||
        L.device_ != L0.device_)
      throw_invalid("grouped linears need one shape, group size, dtype and device");
    if (c.ldx < L.K_ || c.ldy < L.N_) throw_invalid("leading dimensions are smaller than the layer");
    if ((reinterpret_cast<uintptr_t>(c.x) & 15) != 0 || (c.ldx % 8) != 0)
      throw_invalid("input rows must be 16-byte aligned (x % 16 == 0 and ldx % 8 == 0)");
    maps.m[i] = plan.rt == L.plan_.rt ? L.wmap_ : L.wmap_rt_[plan.rt == 1 ? 0 : plan.rt == 2 ? 1 : 2];
    cq::GemvArgs& a = g.a[i];
    a.x = c.x;
    a.scales = L.scales_;
    a.biases = L.biases_;
    a.bias = L.bias_;
    a.y = c.y;
    a.status = ctx.status;
    a.M = rows;
    a.N = L.N_;
    a.K = L.K_;
    a.ldx = c.ldx;
    a.ldy = c.ldy;
    a.sb_per_cta = L.plan_.sb_per_cta;
    a.act = act;
  }
  check_cuda(cq::launch_gemv_group(L0.dtype_, L0.group_, plan, maps, g, stream, pdl_enabled()),
             "qgemv group");
}

void QuantizedLinear::forward_f32(const float* input, size_t input_len, int rows, float* output,
                                  size_t output_len) {
  if (rows < 0 || static_cast<size_t>(rows) * static_cast<size_t>(K_) != input_len)
    throw_invalid("invalid model shape: linear input has " + std::to_string(input_len) +
                  " values, expected " + std::to_string(rows) + "x" + std::to_string(K_));
  if (static_cast<size_t>(rows) * static_cast<size_t>(N_) != output_len)
    throw_invalid("invalid model shape: linear output has " + std::to_string(output_len) +
                  " values, expected " + std::to_string(rows) + "x" + std::to_string(N_));
  if (rows == 0) return;
  if (input == nullptr || output == nullptr) throw_invalid("input and output must not be null");
  std::lock_guard<std::mutex> lock(host_mu_);
  DeviceContext& ctx = device_context(device_);
  DeviceGuard guard(device_);
  const size_t es = dtype_size(dtype_);
  const size_t xin = align_up(input_len * sizeof(float), 256);
  const size_t xt = align_up(input_len * es, 256);
  const size_t yt = align_up(output_len * es, 256);
  const size_t yout = align_up(output_len * sizeof(float), 256);
  const size_t need = xin + xt + yt + yout;
  if (need > host_scratch_bytes_) {
    cudaFree(host_scratch_);
    host_scratch_ = nullptr;
    host_scratch_bytes_ = 0;
    check_cuda(cudaMalloc(&host_scratch_, need), "cudaMalloc(host scratch)");
    host_scratch_bytes_ = need;
  }
  char* base = static_cast<char*>(host_scratch_);
  float* d_xin = reinterpret_cast<float*>(base);
  void* d_xt = base + xin;
  void* d_yt = base + xin + xt;
  float* d_yout = reinterpret_cast<float*>(base + xin + xt + yt);
  cudaStream_t s = cudaStreamPerThread;
  check_cuda(cudaMemcpyAsync(d_xin, input, input_len * sizeof(float), cudaMemcpyHostToDevice, s),
             "upload input");
  if (dtype_ == CQ_F32) {
    forward_array(d_xin, K_, rows, d_yout, N_, CQ_ACT_NONE, s);
  } else {
    check_cuda(cq::launch_f32_to_t(dtype_, d_xin, input_len, d_xt, s), "cast input");
    forward_array(d_xt, K_, rows, d_yt, N_, CQ_ACT_NONE, s);
    check_cuda(cq::launch_t_to_f32(dtype_, d_yt, output_len, d_yout, s), "widen output");
  }
  check_cuda(cudaMemcpyAsync(output, d_yout, output_len * sizeof(float), cudaMemcpyDeviceToHost, s),
             "download output");
  int status = 0;
  check_cuda(cudaMemcpyAsync(&status, ctx.status, sizeof(int), cudaMemcpyDeviceToHost, s),
             "read device status");
  check_cuda(cudaStreamSynchronize(s), "forward_f32");
  if (status != 0)
    throw Error(CQ_RUNTIME_ERROR, "device watchdog: a kernel gave up waiting (status " +
                                      std::to_string(status) + ")");
}

// ------------------------------------------------------------------ backend

void quantized_matmul(const float* input, size_t input_len, size_t rows, size_t input_dims,
                      const float* weight, size_t weight_len, size_t output_dims,
                      size_t group_size, float* output, size_t output_len) {
  // Validation order and texts of backend::quantized_matmul
  // (crates/nemotron-mlx/src/backend/mod.rs:49-75).
  const char* P = "invalid matrix shape: ";
  if (rows * input_dims != input_len || (input_dims != 0 && (rows * input_dims) / input_dims != rows))
    throw_invalid(fmt_shape_error(P, "input has " + std::to_string(input_len) +
                                         " values, expected " + std::to_string(rows) + "x" +
                                         std::to_string(input_dims)));
  if (output_dims * input_dims != weight_len)
    throw_invalid(fmt_shape_error(P, "weight has " + std::to_string(weight_len) +
                                         " values, expected " + std::to_string(output_dims) +
                                         "x" + std::to_string(input_dims)));
  if (group_size == 0) throw_invalid(fmt_shape_error(P, "group size must be positive"));
  if (input_dims % group_size != 0)
    throw_invalid(fmt_shape_error(P, "input dimension " + std::to_string(input_dims) +
                                         " is not divisible by group size " +
                                         std::to_string(group_size)));
  validate_group(static_cast<int>(group_size));
  if (output_len != rows * output_dims)
    throw_invalid(fmt_shape_error(P, "output has " + std::to_string(output_len) +
                                         " values, expected " + std::to_string(rows) + "x" +
                                         std::to_string(output_dims)));
  if (rows == 0 || output_dims == 0) return;
  if (input == nullptr || weight == nullptr || output == nullptr)
    throw_invalid("input, weight and output must not be null");
  int device = 0;
  check_cuda(cudaGetDevice(&device), "cudaGetDevice");
  device_context(device);
  const size_t groups = output_dims * (input_dims / group_size);
  char* buf = nullptr;
  const size_t o_w = 0;
  const size_t o_x = align_up(o_w + weight_len * 4, 256);
  const size_t o_q = align_up(o_x + input_len * 4, 256);
  const size_t o_s = align_up(o_q + weight_len, 256);
  const size_t o_b = align_up(o_s + groups * 4, 256);
  const size_t o_y = align_up(o_b + groups * 4, 256);
  const size_t total = o_y + output_len * 4;
  check_cuda(cudaMalloc(&buf, total), "cudaMalloc(quantized_matmul)");
  float* dw = reinterpret_cast<float*>(buf + o_w);
  float* dx = reinterpret_cast<float*>(buf + o_x);
  uint8_t* dq = reinterpret_cast<uint8_t*>(buf + o_q);
  float* ds = reinterpret_cast<float*>(buf + o_s);
  float* db = reinterpret_cast<float*>(buf + o_b);
  float* dy = reinterpret_cast<float*>(buf + o_y);
  cudaStream_t s = cudaStreamPerThread;
  cudaError_t e = cudaMemcpyAsync(dw, weight, weight_len * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dx, input, input_len * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cq::launch_quantize(CQ_F32, dw, static_cast<int>(output_dims), static_cast<int>(input_dims),
                            static_cast<int>(group_size), false, dq, ds, db, s);
  if (e == cudaSuccess)
    e = cq::launch_qmatmul_f32(dx, static_cast<int>(rows), static_cast<int>(input_dims), dq, ds, db,
                               static_cast<int>(output_dims), static_cast<int>(group_size), dy, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(output, dy, output_len * 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(buf);
  check_cuda(e, "quantized_matmul");
}

}  // namespace nemotron_cuda
