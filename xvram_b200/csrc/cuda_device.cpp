// cuda_device.cpp -- Device implementation over the CUDA runtime and driver VMM API.
//
// Replaces the reference's dynamically loaded driver table (reference
// src/platform/cuda/cuda_api.hpp:30-80).  Driver entry points are resolved through
// cudaGetDriverEntryPoint, so the library links only the static CUDA runtime.  The
// runtime's primary context of the selected device is used: it is shared with any
// other CUDA user in the process (PyTorch, NCCL), which is what lets callers mix the
// adapter with their own device work.
#include "device.hpp"
#include "xvram_b200.h"
#include "kernels.hpp"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

namespace xvram {
namespace {

struct DriverTable {
  decltype(&cuMemAddressReserve) address_reserve = nullptr;
  decltype(&cuMemAddressFree) address_free = nullptr;
  decltype(&cuMemCreate) create = nullptr;
  decltype(&cuMemRelease) release = nullptr;
  decltype(&cuMemMap) map = nullptr;
  decltype(&cuMemUnmap) unmap = nullptr;
  decltype(&cuMemSetAccess) set_access = nullptr;
  decltype(&cuMemGetAllocationGranularity) granularity = nullptr;
  decltype(&cuGetErrorName) error_name = nullptr;
  bool ok = false;
};

template <class F> bool resolve(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !p)
    return false;
  fn = reinterpret_cast<F>(p);
  return true;
}

const DriverTable& driver() {
  static const DriverTable t = [] {
    DriverTable d;
    d.ok = resolve("cuMemAddressReserve", d.address_reserve) &&
           resolve("cuMemAddressFree", d.address_free) && resolve("cuMemCreate", d.create) &&
           resolve("cuMemRelease", d.release) && resolve("cuMemMap", d.map) &&
           resolve("cuMemUnmap", d.unmap) && resolve("cuMemSetAccess", d.set_access) &&
           resolve("cuMemGetAllocationGranularity", d.granularity) &&
           resolve("cuGetErrorName", d.error_name);
    return d;
  }();
  return t;
}

Error rt_error(const char* op, cudaError_t e) {
  return cuda_error("cuda_runtime", op, static_cast<int>(e), cudaGetErrorName(e),
                    cudaGetErrorString(e));
}

Error drv_error(const char* op, CUresult r) {
  const char* name = nullptr;
  if (driver().error_name)
    driver().error_name(r, &name);
  return cuda_error("cuda_driver", op, static_cast<int>(r), name ? name : "CUresult",
                    "driver call failed");
}

#define XV_RT(op, call)                                                                            \
  do {                                                                                             \
    const cudaError_t xv_e = (call);                                                               \
    if (xv_e != cudaSuccess)                                                                       \
      return rt_error(op, xv_e);                                                                   \
  } while (0)

#define XV_DRV(op, call)                                                                           \
  do {                                                                                             \
    const CUresult xv_r = (call);                                                                  \
    if (xv_r != CUDA_SUCCESS)                                                                      \
      return drv_error(op, xv_r);                                                                  \
  } while (0)

class CudaDevice final : public Device {
public:
  Error open(int ordinal, DeviceInfo* info) override {
    int count = 0;
    XV_RT("cudaGetDeviceCount", cudaGetDeviceCount(&count));
    if (ordinal < 0 || ordinal >= count)
      return make_error(XVRAM_STATUS_UNAVAILABLE, "device", "open", "device ordinal out of range");
    XV_RT("cudaSetDevice", cudaSetDevice(ordinal));
    XV_RT("cudaFree(0)", cudaFree(nullptr)); // make the primary context current
    if (!driver().ok)
      return make_error(XVRAM_STATUS_UNAVAILABLE, "device", "open",
                        "CUDA driver VMM entry points are unavailable");
    cudaDeviceProp prop{};
    XV_RT("cudaGetDeviceProperties", cudaGetDeviceProperties(&prop, ordinal));
    if (prop.major < 10)
      return make_error(XVRAM_STATUS_UNSUPPORTED, "device", "open",
                        "this build targets sm_100a (B200) devices");
    ordinal_ = ordinal;
    CUmemAllocationProp p = alloc_prop();
    size_t gran = 0;
    XV_DRV("cuMemGetAllocationGranularity",
           driver().granularity(&gran, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED));
    int driver_version = 0;
    cudaDriverGetVersion(&driver_version);
    info->ordinal = ordinal;
    info->device_count = count;
    info->name = prop.name;
    info->total_bytes = prop.totalGlobalMem;
    info->sm_count = prop.multiProcessorCount;
    info->vmm_granularity = gran;
    info->driver_version = driver_version;
    info->cc_major = prop.major;
    info->cc_minor = prop.minor;
    return {};
  }

  Error close() override {
    for (auto& e : events_)
      if (e)
        cudaEventDestroy(e);
    for (auto& s : streams_)
      if (s)
        cudaStreamDestroy(s);
    events_.clear();
    streams_.clear();
    return {};
  }

  Error mem_get_info(uint64_t* free_bytes, uint64_t* total_bytes) override {
    XV_RT("cudaSetDevice", cudaSetDevice(ordinal_));
    size_t f = 0, t = 0;
    XV_RT("cudaMemGetInfo", cudaMemGetInfo(&f, &t));
    *free_bytes = f;
    *total_bytes = t;
    return {};
  }

  Error va_reserve(uint64_t bytes, uint64_t* va) override {
    CUdeviceptr p = 0;
    XV_DRV("cuMemAddressReserve", driver().address_reserve(&p, bytes, 0, 0, 0));
    *va = static_cast<uint64_t>(p);
    return {};
  }
  Error va_free(uint64_t va, uint64_t bytes) override {
    XV_DRV("cuMemAddressFree", driver().address_free(static_cast<CUdeviceptr>(va), bytes));
    return {};
  }
  Error handle_create(uint64_t bytes, uint64_t* handle) override {
    CUmemAllocationProp p = alloc_prop();
    CUmemGenericAllocationHandle h = 0;
    const CUresult r = driver().create(&h, bytes, &p, 0);
    if (r == CUDA_ERROR_OUT_OF_MEMORY) {
      Error e = drv_error("cuMemCreate", r);
      e.status = XVRAM_STATUS_DEVICE_OUT_OF_MEMORY;
      return e;
    }
    XV_DRV("cuMemCreate", r);
    *handle = static_cast<uint64_t>(h);
    return {};
  }
  Error handle_release(uint64_t handle) override {
    XV_DRV("cuMemRelease", driver().release(static_cast<CUmemGenericAllocationHandle>(handle)));
    return {};
  }
  Error map(uint64_t va, uint64_t bytes, uint64_t handle) override {
    XV_DRV("cuMemMap", driver().map(static_cast<CUdeviceptr>(va), bytes, 0,
                                    static_cast<CUmemGenericAllocationHandle>(handle), 0));
    CUmemAccessDesc access{};
    access.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    access.location.id = ordinal_;
    access.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    const CUresult r = driver().set_access(static_cast<CUdeviceptr>(va), bytes, &access, 1);
    if (r != CUDA_SUCCESS) {
      driver().unmap(static_cast<CUdeviceptr>(va), bytes);
      return drv_error("cuMemSetAccess", r);
    }
    return {};
  }
  Error unmap(uint64_t va, uint64_t bytes) override {
    XV_DRV("cuMemUnmap", driver().unmap(static_cast<CUdeviceptr>(va), bytes));
    return {};
  }

  Error host_alloc(uint64_t bytes, void** out) override {
    XV_RT("cudaSetDevice", cudaSetDevice(ordinal_));
    void* p = nullptr;
    const cudaError_t e = cudaHostAlloc(&p, bytes, cudaHostAllocPortable);
    if (e != cudaSuccess) {
      cudaGetLastError();
      Error err = rt_error("cudaHostAlloc", e);
      err.status = XVRAM_STATUS_HOST_OUT_OF_MEMORY;
      return err;
    }
    *out = p;
    return {};
  }
  Error host_free(void* p) override {
    XV_RT("cudaFreeHost", cudaFreeHost(p));
    return {};
  }

  Error stream_create(StreamId* out) override {
    XV_RT("cudaSetDevice", cudaSetDevice(ordinal_));
    cudaStream_t s = nullptr;
    XV_RT("cudaStreamCreateWithFlags", cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    streams_.push_back(s);
    *out = streams_.size();
    return {};
  }
  Error stream_destroy(StreamId id) override {
    if (id == 0 || id > streams_.size() || !streams_[id - 1])
      return make_error(XVRAM_STATUS_INTERNAL, "device", "stream_destroy", "unknown stream");
    XV_RT("cudaStreamDestroy", cudaStreamDestroy(streams_[id - 1]));
    streams_[id - 1] = nullptr;
    return {};
  }
  Error stream_sync(StreamId id) override {
    XV_RT("cudaStreamSynchronize", cudaStreamSynchronize(stream(id)));
    return {};
  }
  Error event_create(EventId* out) override {
    XV_RT("cudaSetDevice", cudaSetDevice(ordinal_));
    cudaEvent_t e = nullptr;
    XV_RT("cudaEventCreate", cudaEventCreate(&e));
    events_.push_back(e);
    *out = events_.size();
    return {};
  }
  Error event_destroy(EventId id) override {
    if (id == 0 || id > events_.size() || !events_[id - 1])
      return make_error(XVRAM_STATUS_INTERNAL, "device", "event_destroy", "unknown event");
    XV_RT("cudaEventDestroy", cudaEventDestroy(events_[id - 1]));
    events_[id - 1] = nullptr;
    return {};
  }
  Error event_record(EventId e, StreamId s) override {
    XV_RT("cudaEventRecord", cudaEventRecord(event(e), stream(s)));
    return {};
  }
  Error stream_wait_event(StreamId s, EventId e) override {
    XV_RT("cudaStreamWaitEvent", cudaStreamWaitEvent(stream(s), event(e), 0));
    return {};
  }
  Error event_sync(EventId e) override {
    XV_RT("cudaEventSynchronize", cudaEventSynchronize(event(e)));
    return {};
  }
  Error event_elapsed_ms(EventId a, EventId b, float* ms) override {
    XV_RT("cudaEventElapsedTime", cudaEventElapsedTime(ms, event(a), event(b)));
    return {};
  }

  Error copy_2d(uint64_t dst, uint64_t dpitch, uint64_t src, uint64_t spitch, uint64_t width,
                uint64_t height, CopyDir dir, StreamId s) override {
    const cudaMemcpyKind kind = dir == CopyDir::h2d   ? cudaMemcpyHostToDevice
                                : dir == CopyDir::d2h ? cudaMemcpyDeviceToHost
                                                      : cudaMemcpyDeviceToDevice;
    if (height == 1 || (dpitch == width && spitch == width)) {
      XV_RT("cudaMemcpyAsync",
            cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src),
                            width * height, kind, stream(s)));
    } else {
      XV_RT("cudaMemcpy2DAsync",
            cudaMemcpy2DAsync(reinterpret_cast<void*>(dst), dpitch,
                              reinterpret_cast<const void*>(src), spitch, width, height, kind,
                              stream(s)));
    }
    return {};
  }

  Error memset_d32(uint64_t dst, uint32_t value, uint64_t count, StreamId s) override {
    if (value != 0)
      return make_error(XVRAM_STATUS_INTERNAL, "device", "memset", "only zero fill is used");
    XV_RT("cudaMemsetAsync",
          cudaMemsetAsync(reinterpret_cast<void*>(dst), 0, count * 4, stream(s)));
    return {};
  }

  Error gemm(const GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n, int64_t k,
             double alpha, uint64_t a, int64_t lda, uint64_t b, int64_t ldb, double beta,
             uint64_t c, int64_t ldc, uint64_t workspace, uint64_t workspace_bytes,
             StreamId s) override {
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
      return make_error(XVRAM_STATUS_INTERNAL, "executor", "gemm", "tile exceeds int32");
    const cudaError_t e =
        gemm_typed(t.ab, t.c, t.compute, op_a, op_b, static_cast<int>(m), static_cast<int>(n),
                   static_cast<int>(k), alpha, reinterpret_cast<const void*>(a), lda,
                   reinterpret_cast<const void*>(b), ldb, beta, reinterpret_cast<void*>(c), ldc,
                   reinterpret_cast<void*>(workspace), workspace_bytes, stream(s));
    if (e != cudaSuccess)
      return rt_error(t.compute == kTf32 ? "sgemm_tf32x3 launch"
                      : t.ab == kFp64    ? "dgemm launch"
                                         : "sgemm_ffma launch",
                      e);
    return {};
  }

  uint64_t gemm_workspace(const GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n,
                          int64_t k) override {
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
      return 0;
    return gemm_typed_workspace_bytes(t.ab, t.c, t.compute, op_a, op_b, static_cast<int>(m),
                                      static_cast<int>(n), static_cast<int>(k));
  }

  Error convert(uint32_t src_type, uint64_t src, int64_t lds, uint32_t dst_type, uint64_t dst,
                int64_t ldd, int64_t rows, int64_t cols, StreamId s) override {
    if (rows > INT32_MAX || cols > INT32_MAX)
      return make_error(XVRAM_STATUS_INTERNAL, "executor", "convert", "block exceeds int32");
    XV_RT("convert_matrix",
          convert_matrix(src_type, reinterpret_cast<const void*>(src), lds, dst_type,
                         reinterpret_cast<void*>(dst), ldd, static_cast<int>(rows),
                         static_cast<int>(cols), stream(s)));
    return {};
  }

  Error gemm_prepare(const GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n, int64_t k,
                     uint64_t a, int64_t lda, uint64_t b, int64_t ldb, uint64_t workspace,
                     uint64_t workspace_bytes, StreamId s, PreparedGemm* out) override {
    if (t.ab != kFp32 || t.c != kFp32 || (t.compute != kStrictFp32 && t.compute != kTf32))
      return make_error(XVRAM_STATUS_INTERNAL, "executor", "gemm_prepare", "FP32 GEMMs only");
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
      return make_error(XVRAM_STATUS_INTERNAL, "executor", "gemm_prepare", "tile exceeds int32");
    SgemmPrepared p;
    XV_RT("sgemm_prepare",
          sgemm_prepare(t.compute == kTf32, op_a, op_b, static_cast<int>(m), static_cast<int>(n),
                        static_cast<int>(k), reinterpret_cast<const float*>(a), lda,
                        reinterpret_cast<const float*>(b), ldb, reinterpret_cast<void*>(workspace),
                        workspace_bytes, stream(s), &p));
    *out = PreparedGemm{};
    out->compute = t.compute;
    if (p.tf32) {
      out->a = reinterpret_cast<uint64_t>(p.a_hi);
      out->a2 = reinterpret_cast<uint64_t>(p.a_lo);
      out->b = reinterpret_cast<uint64_t>(p.b_hi);
      out->b2 = reinterpret_cast<uint64_t>(p.b_lo);
      out->lda = out->ldb = p.kp;
    } else {
      out->a = reinterpret_cast<uint64_t>(p.a);
      out->b = reinterpret_cast<uint64_t>(p.b);
      out->lda = p.lda;
      out->ldb = p.ldb;
      out->op_a = p.op_a;
      out->op_b = p.op_b;
    }
    return {};
  }

  Error gemm_block(const PreparedGemm& q, int64_t m, int64_t n0, int64_t nj, int64_t k,
                   double alpha, double beta, uint64_t c, int64_t ldc, StreamId s) override {
    if (m > INT32_MAX || n0 + nj > INT32_MAX || k > INT32_MAX)
      return make_error(XVRAM_STATUS_INTERNAL, "executor", "gemm_block", "tile exceeds int32");
    SgemmPrepared p;
    p.tf32 = q.compute == kTf32;
    if (p.tf32) {
      p.a_hi = reinterpret_cast<const float*>(q.a);
      p.a_lo = reinterpret_cast<const float*>(q.a2);
      p.b_hi = reinterpret_cast<const float*>(q.b);
      p.b_lo = reinterpret_cast<const float*>(q.b2);
      p.kp = q.lda;
    } else {
      p.a = reinterpret_cast<const float*>(q.a);
      p.b = reinterpret_cast<const float*>(q.b);
      p.lda = q.lda;
      p.ldb = q.ldb;
      p.op_a = q.op_a;
      p.op_b = q.op_b;
    }
    const cudaError_t e = sgemm_block(p, static_cast<int>(m), static_cast<int>(n0),
                                      static_cast<int>(nj), static_cast<int>(k),
                                      static_cast<float>(alpha), static_cast<float>(beta),
                                      reinterpret_cast<float*>(c), ldc, stream(s));
    if (e != cudaSuccess)
      return rt_error(p.tf32 ? "sgemm_tf32x3 launch" : "sgemm_ffma launch", e);
    return {};
  }

  Error kernel_status(StreamId s, uint32_t* word) override {
    unsigned int w = 0, wt = 0;
    XV_RT("read_kernel_error", read_and_clear_kernel_error(&w, stream(s)));
    XV_RT("read_kernel_error_tc", read_and_clear_kernel_error_tc(&wt, stream(s)));
    *word = w | (wt << 8);
    return {};
  }

  uint64_t native_stream(StreamId s) override { return reinterpret_cast<uint64_t>(stream(s)); }

  Error make_current(int* previous) override {
    XV_RT("cudaGetDevice", cudaGetDevice(previous));
    XV_RT("cudaSetDevice", cudaSetDevice(ordinal_));
    return {};
  }
  void restore_current(int previous) override { cudaSetDevice(previous); }

  Error mem_alloc(uint64_t bytes, uint64_t* out) override {
    XV_RT("cudaSetDevice", cudaSetDevice(ordinal_));
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      Error err = rt_error("cudaMalloc", e);
      if (e == cudaErrorMemoryAllocation)
        err.status = XVRAM_STATUS_DEVICE_OUT_OF_MEMORY;
      return err;
    }
    *out = reinterpret_cast<uint64_t>(p);
    return {};
  }
  Error mem_free(uint64_t p) override {
    XV_RT("cudaFree", cudaFree(reinterpret_cast<void*>(p)));
    return {};
  }

  Error event_query(EventId e, bool* done) override {
    const cudaError_t q = cudaEventQuery(event(e));
    if (q == cudaErrorNotReady) {
      *done = false;
      return {};
    }
    XV_RT("cudaEventQuery", q);
    *done = true;
    return {};
  }

  Error transpose_f32(uint64_t src, int64_t lds, uint64_t dst, int64_t ldd, int64_t rows,
                      int64_t cols, StreamId s) override {
    if (rows > INT32_MAX || cols > INT32_MAX)
      return make_error(XVRAM_STATUS_INTERNAL, "executor", "transpose", "block exceeds int32");
    XV_RT("transpose_f32", transpose_f32_async(reinterpret_cast<const float*>(src), lds,
                                               reinterpret_cast<float*>(dst), ldd,
                                               static_cast<int>(rows), static_cast<int>(cols),
                                               stream(s)));
    return {};
  }

private:
  static CUmemAllocationProp alloc_prop_for(int ordinal) {
    CUmemAllocationProp p{};
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = ordinal;
    return p;
  }
  CUmemAllocationProp alloc_prop() const { return alloc_prop_for(ordinal_); }
  cudaStream_t stream(StreamId id) const {
    return (id == 0 || id > streams_.size()) ? nullptr : streams_[id - 1];
  }
  cudaEvent_t event(EventId id) const {
    return (id == 0 || id > events_.size()) ? nullptr : events_[id - 1];
  }

  int ordinal_ = 0;
  std::vector<cudaStream_t> streams_;
  std::vector<cudaEvent_t> events_;
};

std::unique_ptr<Device> default_factory() { return std::make_unique<CudaDevice>(); }

} // namespace

std::unique_ptr<Device> make_cuda_device() { return std::make_unique<CudaDevice>(); }

DeviceFactory& device_factory() {
  static DeviceFactory f = &default_factory;
  return f;
}

namespace {
void* (*g_external_factory)(void) = nullptr;
std::unique_ptr<Device> external_factory() {
  return std::unique_ptr<Device>(static_cast<Device*>(g_external_factory ? g_external_factory()
                                                                         : nullptr));
}
} // namespace

} // namespace xvram

extern "C" XVRAM_B200_API xvram_status XVRAM_CALL
xvram_b200_device_query(int32_t ordinal, xvram_b200_device_info_v1* out) {
  if (!out || out->struct_size < sizeof(xvram_b200_device_info_v1))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  std::unique_ptr<xvram::Device> dev = xvram::device_factory()();
  if (!dev)
    return XVRAM_STATUS_UNAVAILABLE;
  xvram::DeviceInfo info;
  if (xvram::Error e = dev->open(ordinal, &info)) {
    (void)dev->close();
    return e.status;
  }
  uint64_t free_bytes = 0, total_bytes = 0;
  const xvram::Error mem = dev->mem_get_info(&free_bytes, &total_bytes);
  (void)dev->close();
  const uint32_t size = out->struct_size;
  *out = xvram_b200_device_info_v1{};
  out->struct_size = size;
  out->ordinal = info.ordinal;
  out->device_count = info.device_count;
  std::snprintf(out->name, sizeof(out->name), "%s", info.name.c_str());
  out->total_bytes = info.total_bytes;
  out->free_bytes = mem ? 0 : free_bytes;
  out->sm_count = info.sm_count;
  out->compute_capability_major = info.cc_major;
  out->compute_capability_minor = info.cc_minor;
  out->vmm_granularity = info.vmm_granularity;
  out->driver_version = info.driver_version;
  out->runtime_headers_version = CUDART_VERSION;
  return XVRAM_STATUS_SUCCESS;
}

extern "C" xvram_status xvram_b200_test_set_device_factory(void* (*create)(void)) {
  xvram::g_external_factory = create;
  xvram::device_factory() = create ? &xvram::external_factory : &xvram::default_factory;
  return XVRAM_STATUS_SUCCESS;
}
