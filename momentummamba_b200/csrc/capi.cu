// Status strings and ABI version of the C interface.
#include <mutex>

#include "mmb_common.cuh"

#define MMB_ABI_VERSION 3

extern "C" const char* mmb_status_string(int status) {
    switch (status) {
        case MMB_OK: return "ok";
        case MMB_ERR_NULL: return "a required pointer is NULL";
        case MMB_ERR_SHAPE: return "a size or stride is out of range";
        case MMB_ERR_ALIGN: return "a pointer or stride breaks the required alignment";
        case MMB_ERR_UNSUPPORTED: return "unsupported configuration";
        case MMB_ERR_WORKSPACE: return "workspace missing";
        case MMB_ERR_LAUNCH: return "CUDA launch failed";
        case MMB_ERR_TIMEOUT: return "a bounded device-side wait timed out";
        default: return "unknown status";
    }
}

extern "C" int mmb_abi_version(void) { return MMB_ABI_VERSION; }

static thread_local cudaError_t g_last_cuda_error = cudaSuccess;

void mmb_record_cuda_error(cudaError_t e) { g_last_cuda_error = e; }

extern "C" const char* mmb_last_error(void) {
    if (g_last_cuda_error == cudaSuccess) return "no CUDA error recorded";
    return cudaGetErrorString(g_last_cuda_error);
}

// ---------------------------------------------------------------------------
// device-side error flag: kernels whose bounded waits give up set it
// ---------------------------------------------------------------------------
static __device__ int g_mmb_device_error;

static std::mutex g_flag_mutex;
static int* g_flag_ptr[MMB_MAX_DEVICES] = {};

int* mmb_device_error_flag() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MMB_MAX_DEVICES) return nullptr;
    std::lock_guard<std::mutex> lock(g_flag_mutex);
    if (!g_flag_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_mmb_device_error) != cudaSuccess) return nullptr;
        g_flag_ptr[dev] = static_cast<int*>(p);
    }
    return g_flag_ptr[dev];
}

extern "C" int mmb_device_status(mmb_stream_t stream) {
    MMB_NVTX("mmb_device_status");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        mmb_record_cuda_error(e);
        return MMB_ERR_LAUNCH;
    }
    int flag = 0;
    e = cudaMemcpyFromSymbol(&flag, g_mmb_device_error, sizeof(int));
    if (e != cudaSuccess) {
        mmb_record_cuda_error(e);
        return MMB_ERR_LAUNCH;
    }
    if (flag) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_mmb_device_error, &zero, sizeof(int));
        return MMB_ERR_TIMEOUT;
    }
    return MMB_OK;
}

// Self-test of the device error path.  One CTA arms an mbarrier for 16 bytes
// of a transaction that never comes -- no copy is issued, so nothing
// asynchronous is outstanding when the CTA leaves -- and waits on it the way the
// tile pipelines do, with at most `polls` polls.  The wait gives up, the CTA
// sets the device error flag (as a pipeline that gave up does) and returns.
__global__ void selftest_wait_kernel(int polls, int* err) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mmb::mbar_init(&bar, 1);
        mmb::mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mmb::mbar_expect_tx(&bar, 16);
    __syncthreads();
    const bool landed = mmb::mbar_wait_polls(&bar, 0, polls);
    if (__syncthreads_or(!landed) && threadIdx.x == 0 && err) atomicOr(err, 1);
}

extern "C" int mmb_selftest_device_wait(int32_t polls, mmb_stream_t stream) {
    MMB_NVTX("mmb_selftest_device_wait");
    if (polls < 1 || polls > 4096) return MMB_ERR_SHAPE;
    int* err = mmb_device_error_flag();
    if (!err) return MMB_ERR_LAUNCH;
    selftest_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(polls, err);
    return mmb_launch_status();
}

// ---------------------------------------------------------------------------
// tensor maps (TMA descriptors) through the driver entry point
// ---------------------------------------------------------------------------
typedef CUresult (*mmb_encode_tiled_fn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                        const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                        const cuuint32_t*, CUtensorMapInterleave,
                                        CUtensorMapSwizzle, CUtensorMapL2promotion,
                                        CUtensorMapFloatOOBfill);

static mmb_encode_tiled_fn encode_fn() {
    static std::once_flag once;
    static mmb_encode_tiled_fn fn = nullptr;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<mmb_encode_tiled_fn>(f);
    });
    return fn;
}

bool mmb_encode_tile_map(CUtensorMap* map, const void* base, int elem_bytes, int64_t dim0,
                         int64_t dim1, int64_t dim2, int64_t stride1, int64_t stride2,
                         int box0, int box1, int swizzle_bytes) {
    mmb_encode_tiled_fn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)dim0, (cuuint64_t)dim1, (cuuint64_t)dim2};
    const cuuint64_t strides[2] = {(cuuint64_t)(stride1 * elem_bytes),
                                   (cuuint64_t)(stride2 * elem_bytes)};
    const cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle sw = swizzle_bytes == MMB_SWZ_128B_ATOM32
                                      ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                  : swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                  : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                        : CU_TENSOR_MAP_SWIZZLE_NONE;
    const CUtensorMapDataType dt =
        elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    return fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
