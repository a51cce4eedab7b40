// murm_kernels.cuh — launcher interfaces between the C ABI layer and the kernels.
#pragma once

#include "murm_common.cuh"

namespace murm {

struct Strides3 {
  int64_t s[3];  // {batch, head, row}, elements
};

template <typename T>
__host__ __device__ __forceinline__ const T* row_ptr(const T* base, Strides3 st, int b, int h, int n) {
  return base + (int64_t)b * st.s[0] + (int64_t)h * st.s[1] + (int64_t)n * st.s[2];
}
template <typename T>
__host__ __device__ __forceinline__ T* row_ptr(T* base, Strides3 st, int b, int h, int n) {
  return base + (int64_t)b * st.s[0] + (int64_t)h * st.s[1] + (int64_t)n * st.s[2];
}

struct FwdPtrs {
  const void* q;  Strides3 qs;
  const void* sk; Strides3 sks;
  const void* sv; Strides3 svs;
  void* out;      Strides3 os;
  int64_t* indices;
  float* weights;
  int slots_f32 = 0;  // sk / sv are fp32 slot state (whatever the dtype of q and out)
};

struct BwdPtrs {
  const void* q;  Strides3 qs;
  const void* go; Strides3 gos;
  const float* gw;
  void* gq;  Strides3 gqs;
  void* gsk; Strides3 gsks;
  void* gsv; Strides3 gsvs;
};

// Sets the calling thread's murm_last_error_message() (murm_capi.cu).
murm_status report_error(murm_status s, const char* msg);

// Launch accounting (murm_profile.cu). Every launch goes through MURM_LAUNCH.
void launch_begin(const char* name, cudaStream_t st);
void launch_end(cudaStream_t st);
#define MURM_LAUNCH(name, kernel, grid, block, smem, stream, ...)        \
  do {                                                                   \
    ::murm::launch_begin(name, stream);                                  \
    kernel<<<grid, block, smem, stream>>>(__VA_ARGS__);                  \
    ::murm::launch_end(stream);                                          \
  } while (0)

// Programmatic dependent launch: the kernel may be scheduled while its predecessor on the
// stream is still running (once every predecessor block has called pdl_trigger() or exited);
// it runs its prologue (barriers, shared memory, TMEM), then pdl_wait() returns once the
// predecessor has completed and its writes are visible. Used by the tensor-core round loops,
// whose kernels all follow that pattern.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
#define MURM_LAUNCH_PDL(name, kernel, grid, block, smem, stream, ...)                \
  do {                                                                               \
    ::murm::launch_begin(name, stream);                                              \
    ::murm::launch_pdl(kernel, dim3(grid), dim3(block), smem, stream, __VA_ARGS__);  \
    ::murm::launch_end(stream);                                                      \
  } while (0)

// A cooperative launch (every block resident at once, so blocks may wait on each other),
// also a programmatic dependent of the previous kernel on the stream.
template <typename... KArgs, typename... Args>
inline void launch_coop_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
#define MURM_LAUNCH_COOP_PDL(name, kernel, grid, block, smem, stream, ...)                \
  do {                                                                                    \
    ::murm::launch_begin(name, stream);                                                   \
    ::murm::launch_coop_pdl(kernel, dim3(grid), dim3(block), smem, stream, __VA_ARGS__);  \
    ::murm::launch_end(stream);                                                           \
  } while (0)
// True when `blocks` blocks of `kernel` can all be resident on the current device at once and
// the device supports cooperative launches (murm_profile.cu; cached per kernel and device).
bool coop_fits(const void* kernel, int threads, int smem, int blocks);

// Opts `kernel` into `bytes` of dynamic shared memory on the current device (murm_profile.cu).
// The attribute belongs to one device's context, so it is tracked per (kernel, device) and only
// raised when a launch needs more than was set before; safe to call from several host threads.
cudaError_t smem_opt_in_raw(const void* kernel, int bytes);
template <typename... A>
inline cudaError_t smem_opt_in(void (*kernel)(A...), size_t bytes) {
  return smem_opt_in_raw(reinterpret_cast<const void*>(kernel), static_cast<int>(bytes));
}

// Shared pieces of the round loop (murm_simt.cu).
template <typename T>
void launch_load_slots(const Geom& g, const FwdPtrs& p, const Saved& sv, cudaStream_t st);
void launch_update_finalize(const Geom& g, int r, const Saved& sv, const FwdScratch& fs, cudaStream_t st);

// Tensor-core forward (murm_tc.cu): fp16/bf16, head_dim 64, row strides that
// are multiples of 8 elements.
bool tc_forward_supported(const Geom& g, int dtype, const FwdPtrs& p);
size_t tc_images_bytes(const Geom& g);
template <typename T>
cudaError_t fwd_tc(const Geom& g, const FwdPtrs& p, const Saved& sv, const FwdScratch& fs, cudaStream_t st);
// Tensor-core backward (murm_tc_bwd.cu): same conditions as the forward.
bool tc_backward_supported(const Geom& g, int dtype, const BwdPtrs& p);
size_t tc_bwd_tables_bytes(const Geom& g);
template <typename T>
cudaError_t bwd_tc(const Geom& g, const BwdPtrs& p, const Saved& sv, const BwdScratch& bs, cudaStream_t st);
// Device error word written by bounded waits in tensor-core kernels.
cudaError_t read_and_clear_device_error(int* code, cudaStream_t st);
constexpr int kErrProbe = 16;  // the error bit of the wait probe (murm_tc.cu)
// One block whose bounded wait on an mbarrier either completes (arrive != 0) or runs out after
// limit_ns and sets kErrProbe (murm_tc.cu).
cudaError_t launch_wait_probe(int arrive, uint64_t limit_ns, cudaStream_t st);

// CUDA-core path (murm_simt.cu): every dtype, head_dim 16/32/64.
template <typename T>
cudaError_t fwd_simt(const Geom& g, const FwdPtrs& p, const Saved& sv, const FwdScratch& fs, cudaStream_t st);
template <typename T>
cudaError_t bwd_simt(const Geom& g, const BwdPtrs& p, const Saved& sv, const BwdScratch& bs, cudaStream_t st);

}  // namespace murm
