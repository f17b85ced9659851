// dvattn_paged_sdpa_noalloc: the paged decode for callers that cannot allocate device
// memory themselves -- for example an engine whose memory pool owns the whole GPU and
// forbids cudaMalloc after start-up, or a plain-C host with no allocator of its own to
// hand us a workspace.  The split-KV scratch (schedule header, per-sequence prefix
// sums, partial outputs) lives in one fixed array below, reserved on every GPU that
// loads this library until the process exits.
#include <mutex>

#include "decode.cuh"

namespace {

// 32 MiB of device scratch: enough for the decode workspace of every configuration
// whose dvattn_paged_sdpa_workspace_size() is at most this (e.g. 32 sequences x 64
// query heads of 128 dims needs about 19 MiB on a 148-SM B200).
constexpr size_t kScratchBytes = size_t(32) << 20;
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// Device address of g_scratch per device.  In host code the name g_scratch is only a
// host-side stand-in for the symbol, so the address is looked up once per device (with
// that device current) and cached.
constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

}  // namespace

namespace dvb {
int noalloc_scratch(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DVATTN_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_scratch) != cudaSuccess || !ptr) return DVATTN_ERR_CUDA;
        g_scratch_ptr[dev] = ptr;
    }
    *out = g_scratch_ptr[dev];
    return DVATTN_OK;
}
}  // namespace dvb

extern "C" size_t dvattn_paged_sdpa_noalloc_max_workspace(void) { return kScratchBytes; }

extern "C" int dvattn_paged_sdpa_noalloc(const dvattn_paged_args* args, dvattn_stream_t stream) {
    int st = dvb::decode_validate(args);
    if (st != DVATTN_OK) return st;
    if (args->W * args->S == 0 || args->Hq == 0) return DVATTN_OK;
    const size_t need = dvb::decode_workspace_size(args);
    if (need == 0) return DVATTN_ERR_CUDA;
    if (need > kScratchBytes) return DVATTN_ERR_WORKSPACE;  // problem too large for the fixed scratch
    void* ws = nullptr;
    st = dvb::noalloc_scratch(&ws);
    if (st != DVATTN_OK) return st;
    // Nothing in the scratch needs to start at zero: the schedule phase rewrites the
    // header and prefix sums, and every partial is written before it is read.
    return dvb::decode_launch(args, ws, kScratchBytes, reinterpret_cast<cudaStream_t>(stream), DVATTN_PHASE_ALL);
}
