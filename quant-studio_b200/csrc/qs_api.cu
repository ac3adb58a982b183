// C ABI of libqsb200 (declared in include/qsb200.h): argument checks, per-device
// state, dispatch to the kernel files.
#include <cuda.h>  // CUcontext (the driver calls themselves are resolved at run time)
#include <mutex>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/qsb200.h"
#include "qs_kernels.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(QS_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

struct TypeInfo {
    int type, qk, bytes, needs_qw;
};

const TypeInfo kTypes[] = {
    {qs::QS_Q4_0, 32, 18, 0},      {qs::QS_Q2_K, 256, 84, 0},      {qs::QS_Q3_K, 256, 110, 0},
    {qs::QS_Q4_K, 256, 144, 0},    {qs::QS_Q5_K, 256, 176, 0},     {qs::QS_Q6_K, 256, 210, 0},
    {qs::QS_IQ2_XXS, 256, 66, 1},  {qs::QS_IQ2_XS, 256, 74, 1},    {qs::QS_IQ3_XXS, 256, 98, 0},
    {qs::QS_IQ3_S, 256, 110, 0},   {qs::QS_IQ2_S, 256, 82, 1},     {qs::QS_IQ4_XS, 256, 136, 0},
    {qs::QS_Q4_1, 32, 20, 0},      {qs::QS_Q5_0, 32, 22, 0},       {qs::QS_Q5_1, 32, 24, 0},
    {qs::QS_Q8_0, 32, 34, 0},
};

const TypeInfo* find_type(int t) {
    for (const auto& ti : kTypes)
        if (ti.type == t) return &ti;
    return nullptr;
}

bool is_iq(int t) {
    return t == qs::QS_IQ2_XXS || t == qs::QS_IQ2_XS || t == qs::QS_IQ2_S || t == qs::QS_IQ3_XXS || t == qs::QS_IQ3_S;
}

constexpr int kMaxDevices = 64;

struct DeviceState {
    bool ready = false;
    int num_sms = 0;
    qs::IqTables* iq = nullptr;
    cudaMemPool_t pool = nullptr;  // scratch of qs_tensor_error; keeps its memory between calls
};

std::mutex g_mu[kMaxDevices];  // one per device: devices come up in parallel
DeviceState g_dev[kMaxDevices];

// Caller holds no lock; the device must be current.
int ensure_device(int device, DeviceState** out) {
    if (device < 0 || device >= kMaxDevices) return fail(QS_EINVAL, "device %d out of range", device);
    std::lock_guard<std::mutex> lk(g_mu[device]);
    DeviceState& d = g_dev[device];
    if (!d.ready) {
        cudaError_t e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        e = qs::iq_tables_create(&d.iq);
        if (e != cudaSuccess) return cuda_fail(e, "uploading the lattice codebooks");
        cudaMemPoolProps props;
        memset(&props, 0, sizeof(props));
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        if ((e = cudaMemPoolCreate(&d.pool, &props)) != cudaSuccess) return cuda_fail(e, "cudaMemPoolCreate");
        uint64_t keep = UINT64_MAX;
        if ((e = cudaMemPoolSetAttribute(d.pool, cudaMemPoolAttrReleaseThreshold, &keep)) != cudaSuccess)
            return cuda_fail(e, "cudaMemPoolSetAttribute");
        d.ready = true;
    }
    *out = &d;
    return QS_OK;
}

// The calling thread's current CUDA context, saved when an entry point starts and put back
// when it returns: a call that runs on the device owning its data (cudaSetDevice) must not
// leave that device current for the caller, nor create a context the caller never had.
// The two driver calls are looked up once through the runtime, so the library does not
// link libcuda directly.
struct CtxFns {
    CUresult (*get)(CUcontext*) = nullptr;
    CUresult (*set)(CUcontext) = nullptr;
};

const CtxFns& ctx_fns() {
    static CtxFns f;
    static std::once_flag once;
    std::call_once(once, [] {
        void* g = nullptr;
        void* s = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &g, cudaEnableDefault, &q1) == cudaSuccess &&
            cudaGetDriverEntryPoint("cuCtxSetCurrent", &s, cudaEnableDefault, &q2) == cudaSuccess &&
            q1 == cudaDriverEntryPointSuccess && q2 == cudaDriverEntryPointSuccess) {
            f.get = reinterpret_cast<CUresult (*)(CUcontext*)>(g);
            f.set = reinterpret_cast<CUresult (*)(CUcontext)>(s);
        }
    });
    return f;
}

class CurrentContextGuard {
public:
    CurrentContextGuard() {
        const CtxFns& f = ctx_fns();
        ok_ = f.get && f.get(&saved_) == CUDA_SUCCESS;
    }
    ~CurrentContextGuard() {
        if (!ok_) return;
        const CtxFns& f = ctx_fns();
        CUcontext now = nullptr;
        if (f.get(&now) == CUDA_SUCCESS && now != saved_) f.set(saved_);
    }
    CurrentContextGuard(const CurrentContextGuard&) = delete;
    CurrentContextGuard& operator=(const CurrentContextGuard&) = delete;

private:
    CUcontext saved_ = nullptr;
    bool ok_ = false;
};

// `p` must be memory of `device` (or managed memory): a pointer into another GPU's memory
// would otherwise reach the kernel and fault there.
int check_on_device(const void* p, int device, const char* what) {
    cudaPointerAttributes pa;
    cudaError_t e = cudaPointerGetAttributes(&pa, p);
    if (e != cudaSuccess) return cuda_fail(e, "cudaPointerGetAttributes");
    if (pa.type == cudaMemoryTypeManaged) return QS_OK;
    if (pa.type != cudaMemoryTypeDevice) return fail(QS_EINVAL, "%s is not device memory", what);
    if (pa.device != device) return fail(QS_EINVAL, "%s is on device %d, the call runs on device %d", what, pa.device, device);
    return QS_OK;
}

}  // namespace

#define QS_API __attribute__((visibility("default")))

extern "C" {

QS_API int qs_version(void) { return QSB200_VERSION; }

QS_API const char* qs_last_error(void) { return g_err; }

QS_API int qs_type_supported(int ggml_type) { return find_type(ggml_type) != nullptr; }

QS_API int qs_type_needs_qw(int ggml_type) {
    const TypeInfo* ti = find_type(ggml_type);
    return ti ? ti->needs_qw : 0;
}

QS_API int qs_block_info(int ggml_type, int* qk, int* block_bytes) {
    const TypeInfo* ti = find_type(ggml_type);
    if (!ti) return fail(QS_ENOTSUP, "ggml type %d is not supported", ggml_type);
    if (qk) *qk = ti->qk;
    if (block_bytes) *block_bytes = ti->bytes;
    return QS_OK;
}

QS_API int qs_row_bytes(int ggml_type, int64_t k, int64_t* out_bytes) {
    const TypeInfo* ti = find_type(ggml_type);
    if (!ti) return fail(QS_ENOTSUP, "ggml type %d is not supported", ggml_type);
    if (k <= 0 || k % ti->qk) return fail(QS_EINVAL, "row length %lld is not a positive multiple of %d", (long long)k, ti->qk);
    if (out_bytes) *out_bytes = k / ti->qk * ti->bytes;
    return QS_OK;
}

QS_API int qs_init(int device) {
    CurrentContextGuard keep;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    DeviceState* d = nullptr;
    return ensure_device(device, &d);
}

}  // extern "C"

namespace {

// Make the device that owns `p` current (the runtime's current device may belong to
// another runtime instance in the process, e.g. the one torch links) and prepare it.
int device_of(const void* p, const char* what, int* device, DeviceState** st) {
    cudaPointerAttributes pa;
    cudaError_t e = cudaPointerGetAttributes(&pa, p);
    if (e != cudaSuccess) return cuda_fail(e, "cudaPointerGetAttributes");
    if (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged)
        return fail(QS_EINVAL, "%s is not device memory", what);
    int cur = -1;
    if ((e = cudaGetDevice(&cur)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur != pa.device && (e = cudaSetDevice(pa.device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    *device = pa.device;
    return ensure_device(pa.device, st);
}

// Checks shared by the decode entry points; fills the kernel call.
int check_decode(int ggml_type, const void* blocks, int64_t blocks_row_bytes, int64_t n_rows, int64_t k,
                 qs::DqCall& c) {
    const TypeInfo* ti = find_type(ggml_type);
    if (!ti) return fail(QS_ENOTSUP, "ggml type %d is not supported", ggml_type);
    if (k <= 0 || k % ti->qk) return fail(QS_EINVAL, "row length %lld is not a positive multiple of %d", (long long)k, ti->qk);
    if (n_rows < 0) return fail(QS_EINVAL, "negative row count");
    const int64_t row_bytes = k / ti->qk * ti->bytes;
    if (blocks_row_bytes < row_bytes)
        return fail(QS_EINVAL, "block row stride %lld < packed row size %lld", (long long)blocks_row_bytes, (long long)row_bytes);
    memset(&c, 0, sizeof(c));
    c.blocks = blocks;
    c.blocks_row_bytes = blocks_row_bytes;
    c.n_rows = n_rows;
    c.k = k;
    return QS_OK;
}

int check_source(const void* x, int x_type, const float* qw) {
    if (x_type != QS_SRC_F32 && x_type != QS_SRC_F16 && x_type != QS_SRC_BF16)
        return fail(QS_EINVAL, "source type %d is not F32/F16/BF16", x_type);
    if (!x) return fail(QS_EINVAL, "null source rows");
    if (((uintptr_t)x & 15) || (qw && ((uintptr_t)qw & 15))) return fail(QS_EINVAL, "x and qw must be 16-byte aligned");
    return QS_OK;
}

}  // namespace

extern "C" {

QS_API int qs_quantize(int ggml_type, const void* src, int src_type, int64_t n_rows, int64_t k, const float* qw,
                void* dst, int64_t dst_row_bytes, void* stream) {
    const TypeInfo* ti = find_type(ggml_type);
    if (!ti) return fail(QS_ENOTSUP, "ggml type %d is not supported", ggml_type);
    if (src_type != QS_SRC_F32 && src_type != QS_SRC_F16 && src_type != QS_SRC_BF16)
        return fail(QS_EINVAL, "source type %d is not F32/F16/BF16", src_type);
    if (k <= 0 || k % ti->qk) return fail(QS_EINVAL, "row length %lld is not a positive multiple of %d", (long long)k, ti->qk);
    if (n_rows < 0) return fail(QS_EINVAL, "negative row count");
    const int64_t row_bytes = k / ti->qk * ti->bytes;
    if (dst_row_bytes < row_bytes) return fail(QS_EINVAL, "dst_row_bytes %lld < packed row size %lld", (long long)dst_row_bytes, (long long)row_bytes);
    if (ti->needs_qw && !qw) return fail(QS_ENOIMAT, "ggml type %d needs importance weights (qw)", ggml_type);
    if (n_rows == 0) return QS_OK;
    if (!src || !dst) return fail(QS_EINVAL, "null src or dst");
    if (((uintptr_t)src & 15) || (qw && ((uintptr_t)qw & 15)))
        return fail(QS_EINVAL, "src and qw must be 16-byte aligned");
    CurrentContextGuard keep;

    // run on the device that owns src (the runtime's current device may belong to another
    // runtime instance in the process, e.g. the one torch links)
    cudaPointerAttributes pa;
    cudaError_t e = cudaPointerGetAttributes(&pa, src);
    if (e != cudaSuccess) return cuda_fail(e, "cudaPointerGetAttributes(src)");
    if (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged)
        return fail(QS_EINVAL, "src is not device memory");
    const int device = pa.device;
    int cur = -1;
    if ((e = cudaGetDevice(&cur)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur != device && (e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    int rc;
    if ((rc = check_on_device(dst, device, "dst")) || (qw && (rc = check_on_device(qw, device, "qw")))) return rc;
    DeviceState* d = nullptr;
    if ((rc = ensure_device(device, &d))) return rc;

    qs::QuantArgs a;
    a.src = src;
    a.src_type = src_type;
    a.n_rows = n_rows;
    a.k = k;
    a.qw = qw;
    a.dst = static_cast<uint8_t*>(dst);
    a.dst_row_bytes = dst_row_bytes;
    a.row_bytes = row_bytes;
    a.nblk_row = k / ti->qk;
    a.nblk = n_rows * a.nblk_row;
    qs::LaunchCtx ctx{static_cast<cudaStream_t>(stream), device, d->num_sms};
    if (is_iq(ggml_type) && (e = qs::iq_tables_ensure(d->iq, ggml_type)) != cudaSuccess)
        return cuda_fail(e, "building lattice tables");
    e = is_iq(ggml_type)             ? qs::launch_iq(ggml_type, a, ctx, d->iq)
        : qs::is_blk32(ggml_type)    ? qs::launch_blk32(ggml_type, a, ctx)
                                     : qs::launch_kquant(ggml_type, a, ctx);
    if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    return QS_OK;
}

QS_API int qs_dequantize(int ggml_type, const void* src, int64_t src_row_bytes, int64_t n_rows, int64_t k, float* dst,
                         int64_t dst_row_stride, void* stream) {
    qs::DqCall c;
    int rc = check_decode(ggml_type, src, src_row_bytes, n_rows, k, c);
    if (rc) return rc;
    if (dst_row_stride < k || dst_row_stride % 4) return fail(QS_EINVAL, "dst_row_stride %lld must be >= k and a multiple of 4", (long long)dst_row_stride);
    if (n_rows == 0) return QS_OK;
    if (!src || !dst) return fail(QS_EINVAL, "null src or dst");
    if ((uintptr_t)dst & 15) return fail(QS_EINVAL, "dst must be 16-byte aligned");
    CurrentContextGuard keep;
    int device;
    DeviceState* d;
    if ((rc = device_of(src, "src", &device, &d))) return rc;
    if ((rc = check_on_device(dst, device, "dst"))) return rc;
    c.dst = dst;
    c.dst_stride = dst_row_stride;
    qs::LaunchCtx ctx{static_cast<cudaStream_t>(stream), device, d->num_sms};
    cudaError_t e = qs::launch_dequant(ggml_type, c, ctx, d->iq);
    return e == cudaSuccess ? QS_OK : cuda_fail(e, "dequantize launch");
}

QS_API int qs_block_error(int ggml_type, const void* blocks, int64_t blocks_row_bytes, const void* x, int x_type,
                          int64_t n_rows, int64_t k, const float* qw, double* err, void* stream) {
    qs::DqCall c;
    int rc = check_decode(ggml_type, blocks, blocks_row_bytes, n_rows, k, c);
    if (rc) return rc;
    if (n_rows == 0) return QS_OK;
    if ((rc = check_source(x, x_type, qw))) return rc;
    if (!blocks || !err) return fail(QS_EINVAL, "null blocks or err");
    if ((uintptr_t)err & 7) return fail(QS_EINVAL, "err must be 8-byte aligned");
    CurrentContextGuard keep;
    int device;
    DeviceState* d;
    if ((rc = device_of(blocks, "blocks", &device, &d))) return rc;
    if ((rc = check_on_device(x, device, "x")) || (qw && (rc = check_on_device(qw, device, "qw"))) ||
        (rc = check_on_device(err, device, "err")))
        return rc;
    c.x = x;
    c.x_type = x_type;
    c.qw = qw;
    c.err = err;
    qs::LaunchCtx ctx{static_cast<cudaStream_t>(stream), device, d->num_sms};
    cudaError_t e = qs::launch_block_error(ggml_type, c, ctx, d->iq);
    return e == cudaSuccess ? QS_OK : cuda_fail(e, "block error launch");
}

QS_API int qs_tensor_error(int ggml_type, const void* blocks, int64_t blocks_row_bytes, const void* x, int x_type,
                           int64_t n_rows, int64_t k, const float* qw, double* out, void* stream) {
    qs::DqCall c;
    int rc = check_decode(ggml_type, blocks, blocks_row_bytes, n_rows, k, c);
    if (rc) return rc;
    if (!out) return fail(QS_EINVAL, "null out");
    if ((uintptr_t)out & 7) return fail(QS_EINVAL, "out must be 8-byte aligned");
    if (n_rows > 0) {
        if ((rc = check_source(x, x_type, qw))) return rc;
        if (!blocks) return fail(QS_EINVAL, "null blocks");
    }
    CurrentContextGuard keep;
    int device;
    DeviceState* d;
    if ((rc = device_of(out, "out", &device, &d))) return rc;
    if (n_rows > 0 && ((rc = check_on_device(blocks, device, "blocks")) || (rc = check_on_device(x, device, "x")) ||
                       (qw && (rc = check_on_device(qw, device, "qw")))))
        return rc;
    c.x = x;
    c.x_type = x_type;
    c.qw = qw;
    qs::LaunchCtx ctx{static_cast<cudaStream_t>(stream), device, d->num_sms};
    const int np = qs::dq_partial_count(ggml_type, n_rows, k, ctx);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* partial = nullptr;
    cudaError_t e = cudaMallocFromPoolAsync(&partial, (size_t)np * 2 * sizeof(double), d->pool, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocFromPoolAsync (partial sums)");
    e = qs::launch_tensor_error(ggml_type, c, static_cast<double*>(partial), np, out, ctx, d->iq);
    cudaError_t ef = cudaFreeAsync(partial, st);
    if (e != cudaSuccess) return cuda_fail(e, "tensor error launch");
    return ef == cudaSuccess ? QS_OK : cuda_fail(ef, "cudaFreeAsync (partial sums)");
}

QS_API int qs_device_fault(int device, int* bits) {
    if (!bits) return fail(QS_EINVAL, "null bits");
    CurrentContextGuard keep;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    unsigned int b = 0;
    if ((e = qs::read_fault_bits(&b, true)) != cudaSuccess) return cuda_fail(e, "reading the fault word");
    *bits = (int)b;
    return QS_OK;
}

static_assert(qs::NA_MAX_PARTIALS == QS_NOALLOC_MAX_PARTIALS, "static scratch size and its public constant differ");

QS_API int qs_tensor_error_noalloc(int ggml_type, const void* blocks, int64_t blocks_row_bytes, const void* x,
                                   int x_type, int64_t n_rows, int64_t k, const float* qw, double* out, void* stream) {
    // allocation-free: no ensure_device (it uploads tables and creates a pool), only the
    // static scratch resolved by noalloc_setup
    qs::DqCall c;
    int rc = check_decode(ggml_type, blocks, blocks_row_bytes, n_rows, k, c);
    if (rc) return rc;
    if (!out) return fail(QS_EINVAL, "null out");
    if ((uintptr_t)out & 7) return fail(QS_EINVAL, "out must be 8-byte aligned");
    if (n_rows > 0) {
        if ((rc = check_source(x, x_type, qw))) return rc;
        if (!blocks) return fail(QS_EINVAL, "null blocks");
    }
    CurrentContextGuard keep;
    cudaPointerAttributes pa;
    cudaError_t e = cudaPointerGetAttributes(&pa, out);
    if (e != cudaSuccess) return cuda_fail(e, "cudaPointerGetAttributes");
    if (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged) return fail(QS_EINVAL, "out is not device memory");
    int cur = -1;
    if ((e = cudaGetDevice(&cur)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur != pa.device && (e = cudaSetDevice(pa.device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    if (n_rows > 0 && ((rc = check_on_device(blocks, pa.device, "blocks")) || (rc = check_on_device(x, pa.device, "x")) ||
                       (qw && (rc = check_on_device(qw, pa.device, "qw")))))
        return rc;
    const qs::NoAllocDevice* d = nullptr;
    if ((e = qs::noalloc_setup(pa.device, &d)) != cudaSuccess) return cuda_fail(e, "static scratch set-up");
    c.x = x;
    c.x_type = x_type;
    c.qw = qw;
    qs::LaunchCtx ctx{static_cast<cudaStream_t>(stream), pa.device, d->num_sms};
    const int need = qs::dq_partial_count(ggml_type, n_rows, k, ctx);
    if (need > QS_NOALLOC_MAX_PARTIALS)
        return fail(QS_EINVAL, "launch needs %d partial sums; the static scratch holds %d", need, QS_NOALLOC_MAX_PARTIALS);
    e = qs::launch_tensor_error_noalloc(ggml_type, c, out, ctx, *d);
    return e == cudaSuccess ? QS_OK : cuda_fail(e, "tensor error launch (static scratch)");
}

}  // extern "C"
