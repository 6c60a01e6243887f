// One expert's SwiGLU that allocates nothing on the device.
//
// Some callers cannot call cudaMalloc: host runtimes that hand every byte of
// device memory to their own arena and forbid allocator calls after start-up,
// or plugin hosts that must not grow the device footprint of the process.
// For them the SwiGLU intermediate (silu(gate x) * up x) and the combine
// weight live in a file-scope __device__ array instead of a cudaMalloc'd
// buffer. Every GPU that loads this library holds the array until the
// process exits.
#include <mutex>
#include <string>
#include <vector>

#include "../../include/swiftlet_cuda.h"
#include "kernels.h"
#include "launch.h"

namespace swl {

// Largest intermediate size (moe_intermediate_size) the shared scratch holds.
constexpr int kNoAllocMaxInter = 16384;
// [0, kNoAllocMaxInter): the intermediate vector; [kNoAllocMaxInter]: the
// combine weight (1.0); [kNoAllocMaxInter + 1]: the status word the kernels
// write when the caller passes none. 64 KiB + 256 B per device.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMaxInter + 64];

// Sets the combine weight and clears the internal status word before the
// expert kernels of one call run.
__global__ void k_noalloc_set_weight() {
  g_noalloc_scratch[kNoAllocMaxInter] = 1.0f;
  reinterpret_cast<int*>(g_noalloc_scratch)[kNoAllocMaxInter + 1] = 0;
}

// Device address of the scratch array, looked up once per device with that
// device current. In host code the array's name is only a host-side stand-in.
static float* noalloc_scratch(int device) {
  static std::mutex mu;
  static std::vector<float*> addr;
  std::lock_guard<std::mutex> lock(mu);
  if (device >= int(addr.size())) addr.resize(size_t(device) + 1, nullptr);
  if (!addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) throw Error(ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    addr[device] = static_cast<float*>(p);
  }
  return addr[device];
}

static QLin affine_of(const swl_affine_matrix* m, const char* what) {
  if (!m || !m->weight || !m->scales || !m->biases) throw Error(ERR_INVALID, std::string("null ") + what + " matrix");
  if (m->bits != 4 && m->bits != 8) throw Error(ERR_UNSUPPORTED, std::string(what) + ": bits must be 4 or 8");
  if (m->group <= 0 || (m->group & (m->group - 1)) || m->cols % m->group || m->group % (m->bits == 4 ? 32 : 16))
    throw Error(ERR_UNSUPPORTED, std::string(what) + ": unsupported group size");
  if (m->scale_dtype < 0 || m->scale_dtype > 2) throw Error(ERR_UNSUPPORTED, std::string(what) + ": bad scale dtype");
  if (m->rows <= 0 || m->cols <= 0) throw Error(ERR_INVALID, std::string(what) + ": empty matrix");
  QLin q;
  q.w = static_cast<const uint8_t*>(m->weight);
  q.s = static_cast<const uint8_t*>(m->scales);
  q.b = static_cast<const uint8_t*>(m->biases);
  q.out = m->rows; q.in = m->cols; q.bits = m->bits; q.gs = m->group; q.dt = m->scale_dtype;
  q.row_bytes = int64_t(m->cols) * m->bits / 8;
  q.srow = m->cols / m->group;
  if (q.row_bytes % 16 || reinterpret_cast<uintptr_t>(q.w) % 16)
    throw Error(ERR_UNSUPPORTED, std::string(what) + ": rows and the weight pointer must be 16-byte aligned");
  const uintptr_t sa = m->scale_dtype == 0 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(q.s) % sa || reinterpret_cast<uintptr_t>(q.b) % sa)
    throw Error(ERR_INVALID, std::string(what) + ": misaligned scales or biases");
  return q;
}

}  // namespace swl

using namespace swl;

extern "C" int swl_expert_swiglu_noalloc(const swl_affine_matrix* gate, const swl_affine_matrix* up,
                                         const swl_affine_matrix* down, const float* d_x, float* d_y,
                                         int32_t* d_status, void* stream) {
  try {
    const QLin g = affine_of(gate, "gate"), u = affine_of(up, "up"), d = affine_of(down, "down");
    if (!d_x || !d_y) throw Error(ERR_INVALID, "null input or output");
    if (reinterpret_cast<uintptr_t>(d_x) % 16) throw Error(ERR_INVALID, "x must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(d_status) % 4) throw Error(ERR_INVALID, "status word must be 4-byte aligned");
    if (u.out != g.out || u.in != g.in || d.in != g.out || d.out != g.in)
      throw Error(ERR_INVALID, "gate/up must be [inter, hidden] and down [hidden, inter]");
    if (g.bits != u.bits || g.bits != d.bits || g.dt != u.dt || g.dt != d.dt || g.gs != u.gs || g.gs != d.gs)
      throw Error(ERR_UNSUPPORTED, "gate, up and down must share bits, group size and scale dtype");
    if (g.out > kNoAllocMaxInter)
      throw Error(ERR_CAPACITY, "intermediate size " + std::to_string(g.out) + " exceeds the no-allocation scratch (" +
                                    std::to_string(kNoAllocMaxInter) + " values)");
    int device = 0;
    SWL_CUDA(cudaGetDevice(&device));
    float* scratch = noalloc_scratch(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    MoeArgs m;
    m.sg = g; m.su = u; m.sd = d;
    m.g.lin = g; m.u.lin = u; m.d.lin = d;  // geometry only: no routed experts
    m.topk = 0;
    m.hmid_stride = (g.out + 31) / 32 * 32;
    m.hmid = scratch;  // fully rewritten by the gate/up kernel before the down kernel reads it
    m.shared_scale = scratch + kNoAllocMaxInter;
    m.x = d_x;
    m.h = d_y;  // the down kernel accumulates: start from zero
    m.pick_ids = nullptr; m.pick_w = nullptr; m.advance_sd = nullptr; m.advance_cursor = nullptr;
    // bit 0 of the status word: a bounded wait for weight copies gave up and
    // y is incomplete; the caller's word if given, else the scratch's own
    m.status = d_status ? d_status : reinterpret_cast<int*>(scratch + kNoAllocMaxInter + 1);
    SWL_CUDA(cudaMemsetAsync(d_y, 0, size_t(d.out) * sizeof(float), st));
    launch(k_noalloc_set_weight, dim3(1), dim3(1), 0, st, false);
    launch_moe_gateup(m, st, false);
    launch_moe_down(m, st, false);
    return SWL_OK;
  } catch (const Error& e) {
    set_last_error(e.what());  // reported by swl_last_error()
    return e.code;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return SWL_ERR_INVALID;
  }
}
