// gemma3_cuda.cu - host side of the C-ABI declared in include/gemma3_cuda.h.
//
// One context = one GPU = one CUDA stream.  The context owns the device KV
// cache of all 34 layers for max_batch sequence slots, the uploaded RoPE
// tables, the per-layer QK-norm gains and the scratch the kernels need
// (fp16 Q/K/V staging for prefill, split-KV partials for decode, device
// copies of host arguments).  Nothing on the compute path falls back to the
// CPU: a failure is reported through the return code.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <mutex>
#include <utility>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <vector>

#include "../../include/gemma3_cuda.h"
#include "attn_kernels.cuh"
#include "decode_tc.cuh"
#include "proj_kernels.cuh"
#include "layer_kernels.cuh"
#include "safetensors.hpp"

using g3::kHeadDim;
using g3::kHeads;
using g3::kKvHeads;
using g3::kWindow;

// ------------------------------------------------------------------ errors
static thread_local char g_err[512] = "";

static int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

#define CU_TRY(expr)                                                                                    \
    do {                                                                                                \
        cudaError_t e_ = (expr);                                                                        \
        if (e_ != cudaSuccess)                                                                          \
            return fail(e_ == cudaErrorMemoryAllocation ? GEMMA3_CUDA_ERR_OUT_OF_MEMORY                 \
                                                        : GEMMA3_CUDA_ERR_GENERATION_FAILED,            \
                        "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__);           \
    } while (0)

extern "C" const char *gemma3_cuda_last_error(void) { return g_err; }

// ------------------------------------------------------------------ NCCL (loaded lazily)
// The library does not link NCCL: a process that already holds one (torch's)
// must not get a second copy.  The few entry points are resolved with dlopen
// the first time a communicator is requested.
typedef struct {
    char internal[128];
} g3NcclUniqueId;
typedef void *g3NcclComm;
struct NcclApi {
    int (*getUniqueId)(g3NcclUniqueId *);
    int (*commInitRank)(g3NcclComm *, int, g3NcclUniqueId, int);
    int (*allGather)(const void *, void *, size_t, int, g3NcclComm, cudaStream_t);
    int (*commDestroy)(g3NcclComm);
    const char *(*getErrorString)(int);
    bool ok = false;
};
static NcclApi g_nccl;
static int nccl_load() {
    if (g_nccl.ok) return 0;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "NCCL not loadable: %s", dlerror());
    g_nccl.getUniqueId = (int (*)(g3NcclUniqueId *))dlsym(h, "ncclGetUniqueId");
    g_nccl.commInitRank = (int (*)(g3NcclComm *, int, g3NcclUniqueId, int))dlsym(h, "ncclCommInitRank");
    g_nccl.allGather = (int (*)(const void *, void *, size_t, int, g3NcclComm, cudaStream_t))dlsym(h, "ncclAllGather");
    g_nccl.commDestroy = (int (*)(g3NcclComm))dlsym(h, "ncclCommDestroy");
    g_nccl.getErrorString = (const char *(*)(int))dlsym(h, "ncclGetErrorString");
    if (!g_nccl.getUniqueId || !g_nccl.commInitRank || !g_nccl.allGather || !g_nccl.commDestroy)
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "NCCL symbols missing");
    g_nccl.ok = true;
    return 0;
}
static const int kNcclFloat32 = 7;  // ncclFloat32 in nccl.h
static const int kNcclInt8 = 0;     // ncclInt8 in nccl.h

// ------------------------------------------------------------------ TMA encode (driver entry point)
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn g_encode = nullptr;
static int load_encode() {
    if (g_encode) return 0;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    CU_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess)
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "cuTensorMapEncodeTiled unavailable");
    g_encode = (EncodeTiledFn)fn;
    return 0;
}
// fp16 tensor [planes][rows][256] (planes stride given), box 64 x 64 x 1,
// 128-byte swizzle.
static int make_map(CUtensorMap *m, const void *base, int rows, size_t plane_stride_elems, int planes) {
    cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)plane_stride_elems * 2};
    cuuint32_t box[3] = {64, 64, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

// The same fp16 planes viewed as 4-D {64 dims, rows, 4 dim-blocks, planes}:
// one box of {64, box_rows, box_blocks} lands in shared memory as
// [block][row][64 dims], each 128-byte row swizzled - the layout of the
// prefill kernel's ring slots.
static int make_map4(CUtensorMap *m, const void *base, int rows, size_t plane_stride_elems, int planes,
                     int box_rows, int box_blocks) {
    cuuint64_t dims[4] = {64, (cuuint64_t)rows, (cuuint64_t)(kHeadDim / 64), (cuuint64_t)planes};
    cuuint64_t strides[3] = {(cuuint64_t)kHeadDim * 2, 128, (cuuint64_t)plane_stride_elems * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)box_rows, (cuuint32_t)box_blocks, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

// A layer's BF16 cache [planes][rows][256] viewed as 4-D {64 dims, rows,
// 4 dim-blocks, planes}: one box {64, 128, 1, 1} is a 16 KB chunk [128
// rows][128 B] (128-byte swizzle) of one plane, the unit decode_tc streams.
static int make_map_kv(CUtensorMap *m, const void *base, int rows, int planes) {
    cuuint64_t dims[4] = {64, (cuuint64_t)rows, (cuuint64_t)(kHeadDim / 64), (cuuint64_t)planes};
    cuuint64_t strides[3] = {(cuuint64_t)kHeadDim * 2, 128, (cuuint64_t)rows * kHeadDim * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)g3::kTcTK, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

// Launch with programmatic stream serialization: the kernel may begin while
// the previous kernel of the stream drains; the decode-path kernels call
// griddepcontrol.wait before touching memory another kernel writes.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ context
struct LayerState {
    void *kv = nullptr;
    CUtensorMap tm_kv;  // BF16 cache: the chunk map decode_tc streams
    int rows = 0;
    int is_global = 0;
    uint16_t *qn = nullptr, *kn = nullptr;
    int use_norm = 0;
    __half *wqkv = nullptr;  // fp16 [4096][2560]: Wq rows 0-2047, Wk 2048-3071, Wv 3072-4095
    __half *wo = nullptr;    // fp16 [2560][2048]
    // the rest of the transformer block (gemma3_cuda_set_layer_weights)
    __half *wgu = nullptr;    // fp16 [20480][2560]: gate rows 0-10239, up 10240-20479
    __half *wdown = nullptr;  // fp16 [2560][10240]
    uint16_t *ln = nullptr;   // BF16 [4][2560]: input, post-attention, pre-FFN, post-FFN norm gains
    int ln_set[4] = {0, 0, 0, 0};
    int block_ready = 0;
};

struct gemma3_cuda_ctx {
    gemma3_cuda_config cfg;
    cudaStream_t stream = nullptr;
    size_t esz = 4;
    int shard_lo = 0, shard_hi = 0;
    std::vector<LayerState> layers;
    float *rope_local = nullptr, *rope_global = nullptr;
    int rope_rows = 0;
    // prefill scratch
    __half *qst = nullptr;                 // [8][max_prefill][256] fp16
    __half *kst = nullptr, *vst = nullptr;  // [4][st_rows][256] fp16
    int st_rows = 0;
    // decode scratch
    unsigned *tickets = nullptr;  // [max_batch][4] split arrival counters (zero between calls)
    float *qdec = nullptr;        // [max_batch][8][256] q from prologue_decode (long-range calls)
    float *partial = nullptr;  // [max_batch][8][kMaxSplit][258]
    float *emit = nullptr;     // [max_batch][8][258]
    float *gather = nullptr;   // [kv_ranks][max_batch][8][258]
    // projection scratch (allocated on first use), rows = tokens
    __half *xb = nullptr;  // [rows][2560] layer input in fp16
    __half *ab = nullptr;  // [rows][2048] attention output in fp16
    float *qkv = nullptr;         // q [rows][2048] | k [rows][1024] | v [rows][1024]
    float *attn = nullptr;        // [rows][2048]
    float *xio = nullptr;         // [rows][2560] x / out of the host-pointer layer calls
    int proj_rows = 0;
    float *pp = nullptr;          // split-K partials
    size_t pp_floats = 0;
    // transformer-block scratch (allocated on first use)
    float *gu = nullptr;          // gate [rows][10240] | up [rows][10240]
    __half *hb = nullptr;         // [rows][10240] gelu(gate) * up
    float *delta = nullptr;       // [rows][2560] attention / MLP output before its norm
    float *xfwd = nullptr;        // [rows][2560] residual stream of the host-pointer forward calls
    int blk_rows = 0;
    uint16_t *wstage = nullptr;   // BF16 weight staging for the device-side fp16 conversion
    size_t wstage_elems = 0;
    // tied embedding (gemma3_cuda_set_embeddings)
    uint16_t *embed = nullptr;    // BF16 [vocab][2560]: exact lookups
    __half *embed16 = nullptr;    // fp16 [vocab_pad][2560], zero rows past vocab: the logits GEMM
    uint16_t *final_ln = nullptr; // BF16 [2560]
    int vocab = 0, vocab_pad = 0;
    float *logits = nullptr;      // [rows][vocab_pad]
    int logit_rows = 0;
    int *tok_dev = nullptr;       // [rows] token ids in, [rows] argmax out (after)
    float *top_dev = nullptr;     // [rows] top-1 logits
    // device copies for the host-pointer entry points
    float *io = nullptr;
    size_t io_rows = 0;
    unsigned *err = nullptr;
    // context-parallel prefill: this rank's partial [T][8][256] + [T][8](m, l),
    // and the gathered partials of all ranks
    float *pf_part = nullptr, *pf_gather = nullptr;
    size_t pf_part_cap = 0;
    unsigned *err_host = nullptr;  // page-locked word the kernels set non-zero when they raise a bit of *err
    long long launches = 0;
    int sm_count = 148;
    int dec_ctas_per_sm = 2;  // resident decode_tc CTAs per SM (occupancy query)
    // prefill piece partials of the balanced local-layer schedule (first use)
    float *pf_scratch = nullptr;
    float2 *pf_ml = nullptr;
    unsigned *pf_tickets = nullptr;
    g3NcclComm comm = nullptr;
    // peer-memory exchange of the context-parallel split (gemma3_cuda_peer_init)
    float *pgather = nullptr;     // own receive buffer [2][kv_ranks][max_batch][8][258]
    unsigned *pflags = nullptr;   // own flags [2][kMaxPeers]
    unsigned *pcounter = nullptr; // grid ticket of merge_partials_push
    float *peer_g[g3::kMaxPeers] = {};
    unsigned *peer_f[g3::kMaxPeers] = {};
    bool peer_ready = false, use_peer = false;
    unsigned xepoch = 0;
    // profiling of the dominant kernels (decode_splitkv = 0, prefill_fa = 1)
    bool prof = false;
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_used = 0;
    struct Span { int kind; size_t e0, e1; double work; };
    std::vector<Span> spans;
};

// Events bracketing one launch of a profiled kernel, with its algorithmic
// work (bytes for decode, FLOPs for prefill).
static size_t prof_event(gemma3_cuda_ctx *c) {
    if (c->ev_used == c->ev_pool.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return (size_t)-1;
        c->ev_pool.push_back(e);
    }
    cudaEventRecord(c->ev_pool[c->ev_used], c->stream);
    return c->ev_used++;
}
static void prof_begin(gemma3_cuda_ctx *c, size_t *e0) { *e0 = c->prof ? prof_event(c) : (size_t)-1; }
static void prof_end(gemma3_cuda_ctx *c, int kind, size_t e0, double work) {
    if (!c->prof || e0 == (size_t)-1) return;
    size_t e1 = prof_event(c);
    if (e1 != (size_t)-1) c->spans.push_back({kind, e0, e1, work});
}

static constexpr int kMaxSplit = 128;
static constexpr int kPartialStride = kHeadDim + 2;

static bool is_global_layer(int l) { return (l + 1) % 6 == 0; }

extern "C" void gemma3_cuda_config_default(gemma3_cuda_config *c) {
    if (!c) return;
    c->num_layers = 34;
    c->num_heads = kHeads;
    c->num_kv_heads = kKvHeads;
    c->head_dim = kHeadDim;
    c->sliding_window = kWindow;
    c->rmsnorm_eps = 1e-6f;
    c->max_context = 8192;
    c->max_batch = 1;
    c->kv_dtype = GEMMA3_CUDA_KV_F32;
    c->device = 0;
    c->max_prefill = 8192;
    c->kv_rank = 0;
    c->kv_ranks = 1;
}

static void ctx_release(gemma3_cuda_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->cfg.device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->comm && g_nccl.ok) g_nccl.commDestroy(c->comm);
    for (int r = 0; r < g3::kMaxPeers; ++r)
        if (r != c->cfg.kv_rank) {
            if (c->peer_g[r]) cudaIpcCloseMemHandle(c->peer_g[r]);
            if (c->peer_f[r]) cudaIpcCloseMemHandle(c->peer_f[r]);
        }
    cudaFree(c->pgather);
    cudaFree(c->pf_scratch);
    cudaFree(c->pf_ml);
    cudaFree(c->pf_tickets);
    cudaFree(c->pflags);
    cudaFree(c->pcounter);
    for (auto &L : c->layers) {
        cudaFree(L.kv);
        cudaFree(L.qn);
        cudaFree(L.kn);
        cudaFree(L.wqkv);
        cudaFree(L.wo);
        cudaFree(L.wgu);
        cudaFree(L.wdown);
        cudaFree(L.ln);
    }
    if (c->err_host) cudaFreeHost(c->err_host);
    cudaFree(c->gu);
    cudaFree(c->hb);
    cudaFree(c->delta);
    cudaFree(c->xfwd);
    cudaFree(c->wstage);
    cudaFree(c->embed);
    cudaFree(c->embed16);
    cudaFree(c->final_ln);
    cudaFree(c->logits);
    cudaFree(c->tok_dev);
    cudaFree(c->top_dev);
    cudaFree(c->xb);
    cudaFree(c->ab);
    cudaFree(c->qkv);
    cudaFree(c->attn);
    cudaFree(c->xio);
    cudaFree(c->pp);
    cudaFree(c->rope_local);
    cudaFree(c->rope_global);
    cudaFree(c->qst);
    cudaFree(c->kst);
    cudaFree(c->vst);
    cudaFree(c->tickets);
    cudaFree(c->qdec);
    cudaFree(c->partial);
    cudaFree(c->emit);
    cudaFree(c->gather);
    cudaFree(c->io);
    cudaFree(c->pf_part);
    cudaFree(c->pf_gather);
    cudaFree(c->err);
    for (auto e : c->ev_pool) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

static int ctx_alloc(gemma3_cuda_ctx *c) {
    const gemma3_cuda_config &k = c->cfg;
    CU_TRY(cudaSetDevice(k.device));
    int major = 0, minor = 0;
    CU_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, k.device));
    CU_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, k.device));
    if (major != 10 || minor != 0)
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "device %d is sm_%d%d; this library is built for sm_100a only",
                    k.device, major, minor);
    CU_TRY(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    CU_TRY(cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, k.device));
    c->esz = k.kv_dtype == GEMMA3_CUDA_KV_BF16 ? 2 : 4;
    const int S = (k.max_context + k.kv_ranks - 1) / k.kv_ranks;
    c->shard_lo = std::min(k.max_context, k.kv_rank * S);
    c->shard_hi = std::min(k.max_context, c->shard_lo + S);
    c->layers.resize(k.num_layers);
    for (int l = 0; l < k.num_layers; ++l) {
        LayerState &L = c->layers[l];
        L.is_global = is_global_layer(l);
        L.rows = L.is_global ? std::max(1, c->shard_hi - c->shard_lo) : kWindow;
        const size_t bytes = (size_t)k.max_batch * 2 * kKvHeads * L.rows * kHeadDim * c->esz;
        CU_TRY(cudaMalloc(&L.kv, bytes));
        CU_TRY(cudaMemsetAsync(L.kv, 0, bytes, c->stream));
        CU_TRY(cudaMalloc(&L.qn, kHeadDim * 2));
        CU_TRY(cudaMalloc(&L.kn, kHeadDim * 2));
    }
    CU_TRY(cudaMalloc(&c->qst, (size_t)kHeads * k.max_prefill * kHeadDim * 2));
    CU_TRY(cudaMalloc(&c->tickets, (size_t)k.max_batch * kKvHeads * sizeof(unsigned)));
    CU_TRY(cudaMalloc(&c->qdec, (size_t)k.max_batch * kHeads * kHeadDim * sizeof(float)));
    CU_TRY(cudaMemsetAsync(c->tickets, 0, (size_t)k.max_batch * kKvHeads * sizeof(unsigned), c->stream));
    CU_TRY(cudaMalloc(&c->partial, (size_t)k.max_batch * kHeads * kMaxSplit * kPartialStride * 4));
    CU_TRY(cudaMalloc(&c->emit, (size_t)k.max_batch * kHeads * kPartialStride * 4));
    CU_TRY(cudaMalloc(&c->gather, (size_t)k.kv_ranks * k.max_batch * kHeads * kPartialStride * 4));
    c->io_rows = std::max(k.max_prefill, k.max_batch);
    CU_TRY(cudaMalloc(&c->io, c->io_rows * (2048 + 1024 + 1024 + 2048) * sizeof(float)));
    // status block [bits][pad][address of err_host] (see g3::raise_status)
    CU_TRY(cudaHostAlloc((void **)&c->err_host, sizeof(unsigned), cudaHostAllocMapped));
    *c->err_host = 0;
    {
        void *mirror = nullptr;
        CU_TRY(cudaHostGetDevicePointer(&mirror, c->err_host, 0));
        unsigned long long blk[2] = {0ull, (unsigned long long)(uintptr_t)mirror};
        CU_TRY(cudaMalloc(&c->err, sizeof blk));
        CU_TRY(cudaMemcpy(c->err, blk, sizeof blk, cudaMemcpyHostToDevice));
    }
    CU_TRY(cudaFuncSetAttribute(g3::prefill_fa_sm100, cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kPfSmem));
    CU_TRY(cudaFuncSetAttribute(g3::proj_gemm_sm100, cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kProjSmem));
    const int dsm_bf = g3::DecodeCfg<__nv_bfloat16>::NS * 2 * g3::DecodeCfg<__nv_bfloat16>::TK * kHeadDim * 2;
    const int dsm_f = g3::DecodeCfg<float>::NS * 2 * g3::DecodeCfg<float>::TK * kHeadDim * 4;
    CU_TRY(cudaFuncSetAttribute(g3::decode_splitkv<__nv_bfloat16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                dsm_bf + g3::kFusedExtra<__nv_bfloat16>));
    CU_TRY(cudaFuncSetAttribute(g3::decode_splitkv<float, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                dsm_f + g3::kFusedExtra<float>));
    CU_TRY(cudaFuncSetAttribute(g3::decode_splitkv<__nv_bfloat16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dsm_bf));
    CU_TRY(cudaFuncSetAttribute(g3::decode_splitkv<float, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dsm_f));
    if (int r = load_encode()) return r;
    if (k.kv_dtype == GEMMA3_CUDA_KV_BF16) {
        for (auto &L : c->layers)
            if (int r = make_map_kv(&L.tm_kv, L.kv, L.rows, k.max_batch * 2 * kKvHeads)) return r;
        CU_TRY(cudaFuncSetAttribute(g3::decode_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kTcSmem));
        CU_TRY(cudaFuncSetAttribute(g3::decode_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kTcSmem));
        CU_TRY(cudaFuncSetAttribute(g3::decode_tc<true, g3::DecodeRowsSmall>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kTcSmem));
        CU_TRY(cudaFuncSetAttribute(g3::decode_tc<false, g3::DecodeRowsSmall>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kTcSmem));
        CU_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c->dec_ctas_per_sm, g3::decode_tc<false>,
                                                             g3::kTcThreads, g3::kTcSmem));
        if (c->dec_ctas_per_sm < 1)
            return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "decode_tc cannot be resident on this device");
    }
    CU_TRY(cudaStreamSynchronize(c->stream));
    return 0;
}

extern "C" gemma3_cuda_ctx *gemma3_cuda_init(const gemma3_cuda_config *cfg) {
    g_err[0] = 0;
    if (!cfg) {
        fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null config");
        return nullptr;
    }
    const gemma3_cuda_config &k = *cfg;
    if (k.num_heads != kHeads || k.num_kv_heads != kKvHeads || k.head_dim != kHeadDim ||
        k.sliding_window != kWindow || k.num_layers <= 0 || k.num_layers > 256 || k.max_context <= 0 ||
        k.max_batch <= 0 || k.max_batch > g3::kMaxDecodeBatch || k.max_prefill <= 0 ||
        (k.kv_dtype != GEMMA3_CUDA_KV_F32 && k.kv_dtype != GEMMA3_CUDA_KV_BF16) || k.kv_ranks < 1 ||
        k.kv_rank < 0 || k.kv_rank >= k.kv_ranks) {
        fail(GEMMA3_CUDA_ERR_INVALID_ARG,
             "unsupported configuration (needs 8 q heads, 4 kv heads, head_dim 256, window 1024, "
             "1 <= max_batch <= %d, valid kv_rank/kv_ranks)",
             g3::kMaxDecodeBatch);
        return nullptr;
    }
    gemma3_cuda_ctx *c = new gemma3_cuda_ctx();
    c->cfg = k;
    if (ctx_alloc(c) != 0) {
        char keep[512];
        memcpy(keep, g_err, sizeof keep);
        ctx_release(c);
        memcpy(g_err, keep, sizeof keep);
        return nullptr;
    }
    return c;
}

extern "C" void gemma3_cuda_free(gemma3_cuda_ctx *ctx) { ctx_release(ctx); }

extern "C" void *gemma3_cuda_stream(gemma3_cuda_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }
extern "C" long long gemma3_cuda_launch_count(gemma3_cuda_ctx *ctx) { return ctx ? ctx->launches : 0; }

extern "C" int gemma3_cuda_synchronize(gemma3_cuda_ctx *ctx) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    CU_TRY(cudaStreamSynchronize(ctx->stream));
    // Kernels that raise a status bit also set the page-locked err_host, so
    // the status itself is copied back only after a failure.
    if (*reinterpret_cast<volatile unsigned *>(ctx->err_host) == 0u) return 0;
    unsigned e = 0;
    CU_TRY(cudaMemcpy(&e, ctx->err, sizeof(unsigned), cudaMemcpyDeviceToHost));
    // an aborted launch may leave split tickets counted: start clean
    cudaMemsetAsync(ctx->tickets, 0, (size_t)ctx->cfg.max_batch * kKvHeads * sizeof(unsigned), ctx->stream);
    if (ctx->pf_tickets) cudaMemsetAsync(ctx->pf_tickets, 0, g3::kPfMaxCtas * sizeof(unsigned), ctx->stream);
    cudaMemsetAsync(ctx->err, 0, sizeof(unsigned), ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    *reinterpret_cast<volatile unsigned *>(ctx->err_host) = 0u;
    return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "device status 0x%x (%s)", e,
                (e & g3::kErrWaitTimeout) ? "bounded wait timed out"
                : (e & g3::kErrRange)     ? "prefill operand outside the fp16 range"
                                          : "bad index");
}

// Host RoPE table, the formula of gemma3_rope_precompute
// (gemma3_kernels.c:455-468): freq = 1/theta^(2i/d), angle = (float)pos*freq.
extern "C" void gemma3_cuda_rope_precompute(float *freqs, int max_pos, int head_dim, float theta) {
    if (!freqs || max_pos <= 0 || head_dim <= 0) return;
    const int half = head_dim / 2;
    std::vector<float> inv(half);
    for (int i = 0; i < half; ++i) inv[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
    for (int p = 0; p < max_pos; ++p)
        for (int i = 0; i < half; ++i) {
            const float a = (float)p * inv[i];
            freqs[((size_t)p * half + i) * 2] = cosf(a);
            freqs[((size_t)p * half + i) * 2 + 1] = sinf(a);
        }
}

extern "C" int gemma3_cuda_upload_rope(gemma3_cuda_ctx *ctx, const float *rope_local, const float *rope_global,
                                       int max_context, int head_dim) {
    if (!ctx || !rope_local || !rope_global) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null argument");
    if (head_dim != kHeadDim || max_context < ctx->cfg.max_context)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "rope table must cover max_context=%d rows of head_dim 256",
                    ctx->cfg.max_context);
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    const size_t n = (size_t)ctx->cfg.max_context * kHeadDim;
    if (!ctx->rope_local) {
        CU_TRY(cudaMalloc(&ctx->rope_local, n * 4));
        CU_TRY(cudaMalloc(&ctx->rope_global, n * 4));
    }
    CU_TRY(cudaMemcpyAsync(ctx->rope_local, rope_local, n * 4, cudaMemcpyHostToDevice, ctx->stream));
    CU_TRY(cudaMemcpyAsync(ctx->rope_global, rope_global, n * 4, cudaMemcpyHostToDevice, ctx->stream));
    CU_TRY(cudaStreamSynchronize(ctx->stream));
    ctx->rope_rows = ctx->cfg.max_context;
    return 0;
}

extern "C" int gemma3_cuda_set_qk_norm(gemma3_cuda_ctx *ctx, int layer, const uint16_t *q_norm,
                                       const uint16_t *k_norm) {
    if (!ctx || layer < 0 || layer >= ctx->cfg.num_layers) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad layer");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    LayerState &L = ctx->layers[layer];
    L.use_norm = (q_norm && k_norm) ? 1 : 0;
    if (L.use_norm) {
        CU_TRY(cudaMemcpyAsync(L.qn, q_norm, kHeadDim * 2, cudaMemcpyHostToDevice, ctx->stream));
        CU_TRY(cudaMemcpyAsync(L.kn, k_norm, kHeadDim * 2, cudaMemcpyHostToDevice, ctx->stream));
        CU_TRY(cudaStreamSynchronize(ctx->stream));
    }
    return 0;
}

static g3::LayerDev layer_dev(gemma3_cuda_ctx *ctx, int layer) {
    const LayerState &L = ctx->layers[layer];
    g3::LayerDev d;
    d.kv = L.kv;
    d.rows = L.rows;
    d.is_global = L.is_global;
    d.shard_lo = L.is_global ? ctx->shard_lo : 0;
    d.shard_hi = L.is_global ? ctx->shard_hi : kWindow;
    d.qn = L.use_norm ? L.qn : nullptr;
    d.kn = L.use_norm ? L.kn : nullptr;
    d.rope = L.is_global ? ctx->rope_global : ctx->rope_local;
    return d;
}

static int check_launch(gemma3_cuda_ctx *ctx, int n) {
    ctx->launches += n;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "kernel launch failed: %s", cudaGetErrorString(e));
    return 0;
}

// ------------------------------------------------------------------ prefill
// One prefill call of T tokens at start_pos.  out [T][2048]; ml null, or
// [T][8] (m, l) per output row (context-parallel partials).  On a global
// layer of a context-parallel context this rank holds positions
// [shard_lo, shard_hi): it appends the call's rows in that range and attends
// every query to its own keys only (rows of queries with none stay 0 with
// l = 0), so the ranks' outputs merge by log-sum-exp.
template <typename KVT>
static int prefill_impl(gemma3_cuda_ctx *ctx, int layer, int seq, const float *Q, const float *K, const float *V,
                        int T, int start_pos, float *out, float2 *ml) {
    g3::LayerDev L = layer_dev(ctx, layer);
    const bool global = ctx->layers[layer].is_global;
    const bool split = global && ctx->cfg.kv_ranks > 1;
    const int kv_pos0 = split ? ctx->shard_lo : global ? 0 : std::max(0, start_pos - (kWindow - 1));
    const int kv_end = split ? std::min(ctx->shard_hi, start_pos + T) : start_pos + T;
    // queries from qa on can see a key of this context (all of them unless split)
    const int qa = split ? std::max(start_pos, kv_pos0) : start_pos;
    const int Tq = kv_end > kv_pos0 ? start_pos + T - qa : 0;
    if (Tq < T) {
        // queries before this rank's first key: no output, l = 0
        const int n0 = T - Tq;
        CU_TRY(cudaMemsetAsync(out, 0, (size_t)n0 * kHeads * kHeadDim * sizeof(float), ctx->stream));
        if (ml) CU_TRY(cudaMemsetAsync(ml, 0, (size_t)n0 * kHeads * sizeof(float2), ctx->stream));
    }
    const int lrows = std::max(0, kv_end - kv_pos0);  // key rows the attention sees
    if (ctx->st_rows < lrows) {
        cudaFree(ctx->kst);
        cudaFree(ctx->vst);
        ctx->kst = ctx->vst = nullptr;
        ctx->st_rows = 0;
        const int want = std::max(lrows, std::min(ctx->cfg.max_context, kWindow - 1 + ctx->cfg.max_prefill));
        CU_TRY(cudaMalloc(&ctx->kst, (size_t)kKvHeads * want * kHeadDim * 2));
        CU_TRY(cudaMalloc(&ctx->vst, (size_t)kKvHeads * want * kHeadDim * 2));
        ctx->st_rows = want;
    }
    const int nprefix = std::min(start_pos, kv_end) - kv_pos0;
    if (nprefix > 0) {
        g3::stage_prefix<KVT><<<dim3(nprefix, 8), 32, 0, ctx->stream>>>(L, seq, kv_pos0, ctx->kst, ctx->vst,
                                                                          ctx->st_rows, ctx->err);
        if (int r = check_launch(ctx, 1)) return r;
    }
    launch_pdl(g3::prologue_prefill<KVT>, dim3(T), dim3(512), 0, ctx->stream, Q, K, V, L, ctx->cfg.rmsnorm_eps, seq,
               T, start_pos, kv_pos0, kv_end, ctx->qst, ctx->kst, ctx->vst, ctx->st_rows, ctx->err);
    if (int r = check_launch(ctx, 1)) return r;
    if (Tq == 0) return 0;

    CUtensorMap tq, tk, tv;
    const size_t plane = (size_t)ctx->st_rows * kHeadDim;
    const int q0 = qa - start_pos;  // first query token attended here
    if (int r = make_map(&tq, ctx->qst + (size_t)q0 * kHeadDim, Tq, (size_t)T * kHeadDim, kHeads)) return r;
    // K: boxes of 128 keys x 2 dim-blocks; V: 64 keys x 4 dim-blocks (32 KB each)
    if (int r = make_map4(&tk, ctx->kst, lrows, plane, kKvHeads, g3::kPfTK, 2)) return r;
    if (int r = make_map4(&tv, ctx->vst, lrows, plane, kKvHeads, 64, 4)) return r;
    g3::PrefillParams p;
    p.out = out + (size_t)q0 * kHeads * kHeadDim;
    p.ml_out = ml ? ml + (size_t)q0 * kHeads : nullptr;
    p.T = Tq;
    p.start_pos = qa;
    p.kv_pos0 = kv_pos0;
    p.kv_end = kv_end;
    p.is_global = global;
    p.err = ctx->err;
    T = Tq;
    start_pos = qa;
    const int nqb = (T + 63) / 64;
    p.nqb = nqb;
    int grid = std::min(nqb * kKvHeads, ctx->sm_count);  // persistent: one CTA per SM
    p.sched = 0;
    p.nfull = 0;
    p.split = 1;
    p.pscratch = ctx->pf_scratch;
    p.pml = ctx->pf_ml;
    p.ptickets = ctx->pf_tickets;
    if (!global) {
        // Local-layer units are near-equal (up to 17 tiles), so whole units
        // in snake rounds leave the last round short of work on most SMs
        // (T = 8192: 512 units on 148 SMs, 3 full rounds and 68 units
        // over: 4 SMs run four 17-tile units, 80 run three).  Schedule 1 of
        // PrefillParams runs the left-over units first, cut into 2-4 pieces
        // spread over the CTAs, and merges each unit's pieces behind the
        // full rounds.
        const int nunits = nqb * kKvHeads;
        const int G = std::min(ctx->sm_count, g3::kPfMaxCtas);
        const int rest = nunits % G;
        const int split = rest > 0 ? std::min(4, G / rest) : 0;
        if (nunits > G && split >= 2) {
            if (!ctx->pf_scratch) {
                CU_TRY(cudaMalloc(&ctx->pf_scratch, (size_t)g3::kPfMaxCtas * 128 * kHeadDim * sizeof(float)));
                CU_TRY(cudaMalloc(&ctx->pf_ml, (size_t)g3::kPfMaxCtas * 128 * sizeof(float2)));
                CU_TRY(cudaMalloc(&ctx->pf_tickets, g3::kPfMaxCtas * sizeof(unsigned)));
                CU_TRY(cudaMemsetAsync(ctx->pf_tickets, 0, g3::kPfMaxCtas * sizeof(unsigned), ctx->stream));
                p.pscratch = ctx->pf_scratch;
                p.pml = ctx->pf_ml;
                p.ptickets = ctx->pf_tickets;
            }
            p.sched = 1;
            p.nfull = nunits - rest;
            p.split = split;
            grid = G;
        }
    }
    size_t e0;
    prof_begin(ctx, &e0);
    launch_pdl(g3::prefill_fa_sm100, dim3(grid), dim3(g3::kPfThreads), g3::kPfSmem, ctx->stream, tq, tk, tv, p);
    if (ctx->prof) {
        // algorithmic FLOPs: 2 (QK) + 2 (PV) x 256 x 8 heads per attended key
        double keys = 0;
        for (int t = 0; t < T; ++t) {
            const int pos = start_pos + t;
            keys += split ? std::min(pos + 1, kv_end) - kv_pos0 : global ? pos + 1 : std::min(pos + 1, kWindow);
        }
        prof_end(ctx, 1, e0, keys * 4.0 * kHeadDim * kHeads);
    }
    return check_launch(ctx, 1);
}

static int prefill_check(gemma3_cuda_ctx *ctx, int layer, int seq, int T, int start_pos) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    if (layer < 0 || layer >= ctx->cfg.num_layers) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad layer %d", layer);
    if (seq < 0 || seq >= ctx->cfg.max_batch) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad sequence slot %d", seq);
    if (T <= 0 || T > ctx->cfg.max_prefill || start_pos < 0)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad token range T=%d start_pos=%d (max_prefill %d)", T, start_pos,
                    ctx->cfg.max_prefill);
    if ((long long)start_pos + T > ctx->cfg.max_context)
        return fail(GEMMA3_CUDA_ERR_CONTEXT_OVERFLOW, "positions up to %d exceed max_context %d", start_pos + T - 1,
                    ctx->cfg.max_context);
    if (!ctx->rope_local) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "RoPE tables not uploaded");
    return 0;
}

static int prefill_dispatch(gemma3_cuda_ctx *ctx, int layer, int seq, const float *Q, const float *K,
                            const float *V, int T, int start_pos, float *out, float2 *ml) {
    if (ctx->cfg.kv_dtype == GEMMA3_CUDA_KV_BF16)
        return prefill_impl<__nv_bfloat16>(ctx, layer, seq, Q, K, V, T, start_pos, out, ml);
    return prefill_impl<float>(ctx, layer, seq, Q, K, V, T, start_pos, out, ml);
}

extern "C" int gemma3_cuda_merge_prefill_partials_dev(gemma3_cuda_ctx *ctx, int n_parts, int T, const float *outs,
                                                      const float *mls, float *out) {
    if (!ctx || n_parts <= 0 || T <= 0 || !outs || !mls || !out)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad argument");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    launch_pdl(g3::merge_prefill_partials, dim3(T * kHeads), dim3(256), 0, ctx->stream, outs,
               (size_t)T * kHeads * kHeadDim, reinterpret_cast<const float2 *>(mls), (size_t)T * kHeads, n_parts,
               out);
    return check_launch(ctx, 1);
}

extern "C" int gemma3_cuda_attn_prefill_partial_dev(gemma3_cuda_ctx *ctx, int layer, int seq, const float *Q,
                                                    const float *K, const float *V, int T, int start_pos,
                                                    float *out, float *ml) {
    if (int r = prefill_check(ctx, layer, seq, T, start_pos)) return r;
    if (!Q || !K || !V || !out || !ml) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    return prefill_dispatch(ctx, layer, seq, Q, K, V, T, start_pos, out, reinterpret_cast<float2 *>(ml));
}

extern "C" int gemma3_cuda_attn_prefill_dev(gemma3_cuda_ctx *ctx, int layer, int seq, const float *Q,
                                            const float *K, const float *V, int T, int start_pos, float *out) {
    if (int r = prefill_check(ctx, layer, seq, T, start_pos)) return r;
    if (!Q || !K || !V || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    if (!(ctx->layers[layer].is_global && ctx->cfg.kv_ranks > 1))
        return prefill_dispatch(ctx, layer, seq, Q, K, V, T, start_pos, out, nullptr);
    // Context-parallel global layer: this rank's partial over its keys, the
    // ranks' partials all-gathered with NCCL, then the log-sum-exp merge.
    if (!ctx->comm)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG,
                    "global layer of a context-parallel context needs gemma3_cuda_comm_init (or the partial API)");
    const int R = ctx->cfg.kv_ranks;
    const size_t part = (size_t)T * kHeads * (kHeadDim + 2);  // floats: outputs, then (m, l) pairs
    if (ctx->pf_part_cap < part) {
        cudaFree(ctx->pf_part);
        cudaFree(ctx->pf_gather);
        ctx->pf_part = ctx->pf_gather = nullptr;
        ctx->pf_part_cap = 0;
        const size_t cap = (size_t)ctx->cfg.max_prefill * kHeads * (kHeadDim + 2);
        CU_TRY(cudaMalloc(&ctx->pf_part, cap * sizeof(float)));
        CU_TRY(cudaMalloc(&ctx->pf_gather, cap * R * sizeof(float)));
        ctx->pf_part_cap = cap;
    }
    float *mine = ctx->pf_part;
    float2 *ml = reinterpret_cast<float2 *>(mine + (size_t)T * kHeads * kHeadDim);
    if (int r = prefill_dispatch(ctx, layer, seq, Q, K, V, T, start_pos, mine, ml)) return r;
    int nr = g_nccl.allGather(mine, ctx->pf_gather, part, kNcclFloat32, ctx->comm, ctx->stream);
    if (nr != 0)
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "ncclAllGather failed: %s",
                    g_nccl.getErrorString ? g_nccl.getErrorString(nr) : "?");
    launch_pdl(g3::merge_prefill_partials, dim3(T * kHeads), dim3(256), 0, ctx->stream, (const float *)ctx->pf_gather,
               part, reinterpret_cast<const float2 *>(ctx->pf_gather + (size_t)T * kHeads * kHeadDim),
               part / 2, R, out);
    return check_launch(ctx, 1);
}

extern "C" int gemma3_cuda_attn_prefill(gemma3_cuda_ctx *ctx, int layer, int seq, const float *Q, const float *K,
                                        const float *V, int T, int start_pos, float *out) {
    if (int r = prefill_check(ctx, layer, seq, T, start_pos)) return r;
    if (!Q || !K || !V || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    float *dq = ctx->io, *dk = dq + (size_t)T * 2048, *dv = dk + (size_t)T * 1024, *dout = dv + (size_t)T * 1024;
    CU_TRY(cudaMemcpyAsync(dq, Q, (size_t)T * 2048 * 4, cudaMemcpyHostToDevice, ctx->stream));
    CU_TRY(cudaMemcpyAsync(dk, K, (size_t)T * 1024 * 4, cudaMemcpyHostToDevice, ctx->stream));
    CU_TRY(cudaMemcpyAsync(dv, V, (size_t)T * 1024 * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (int r = gemma3_cuda_attn_prefill_dev(ctx, layer, seq, dq, dk, dv, T, start_pos, dout)) return r;
    CU_TRY(cudaMemcpyAsync(out, dout, (size_t)T * 2048 * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return gemma3_cuda_synchronize(ctx);
}

// ------------------------------------------------------------------ decode
struct DecodePlan {
    g3::DecodeRows rows;
    int chunk = 0, nsplit = 0;
};

static int decode_check(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids, const int *pos) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    if (layer < 0 || layer >= ctx->cfg.num_layers) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad layer %d", layer);
    if (B <= 0 || B > ctx->cfg.max_batch || !seq_ids || !pos)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad batch B=%d (max_batch %d)", B, ctx->cfg.max_batch);
    if (!ctx->rope_local) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "RoPE tables not uploaded");
    uint64_t seen[g3::kMaxDecodeBatch / 64] = {};  // max_batch <= kMaxDecodeBatch (checked at init)
    for (int b = 0; b < B; ++b) {
        const int s = seq_ids[b];
        if (s < 0 || s >= ctx->cfg.max_batch || ((seen[s >> 6] >> (s & 63)) & 1u))
            return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad or repeated sequence slot %d", s);
        seen[s >> 6] |= 1ull << (s & 63);
        if (pos[b] < 0) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "negative position");
        if (pos[b] >= ctx->cfg.max_context)
            return fail(GEMMA3_CUDA_ERR_CONTEXT_OVERFLOW, "position %d >= max_context %d", pos[b], ctx->cfg.max_context);
    }
    return 0;
}

template <typename KVT>
static void plan_decode(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids, const int *pos, DecodePlan &pl) {
    const LayerState &L = ctx->layers[layer];
    // tile rows: decode_tc streams 128-row tiles (BF16), decode_splitkv
    // 16-row tiles (fp32); a split holds whole tiles except for its last
    constexpr bool kTc = std::is_same<KVT, __nv_bfloat16>::value;
    constexpr int TK = kTc ? g3::kTcTK : g3::DecodeCfg<KVT>::TK;
    constexpr int kMinTiles = kTc ? 1 : 2;
    pl.rows.B = B;
    int maxrows = 0;
    for (int b = 0; b < B; ++b) {
        pl.rows.seq[b] = seq_ids[b];
        pl.rows.pos[b] = pos[b];
        int n;
        if (L.is_global) {
            n = std::min(pos[b] + 1, ctx->shard_hi) - ctx->shard_lo;
            n = std::max(0, std::min(n, L.rows));
        } else {
            n = std::min(pos[b] + 1, kWindow);
        }
        pl.rows.nrows[b] = n;
        maxrows = std::max(maxrows, n);
    }
    // Rows per split from a cost model of the split kernel, calibrated on
    // B200 measurements.  Two CTAs are resident per SM; each streams its K/V
    // rows at ~22.6 GB/s (all 2 x SMs slots together saturate HBM) and pays
    // a fixed ~4 us (launch, first-copy latency, prologue) plus ~2 us when
    // its result is a partial to merge.  Splits of one call are near equal,
    // so they run in waves: a call of N CTAs takes ceil(N / slots) CTA
    // times, where a unit's last split shorter than a quarter split is not
    // counted (it ends within its wave).  The model picks, e.g., B=8 x 1024
    // local rows: 8 splits of 128 (one wave); B=64 x 1024: one split each;
    // B=64 x 32K global rows: splits of ~4K rows (7 full waves).  Splits hold
    // at least 2 tiles, and a unit at most kMaxSplit.
    const int units = B * kKvHeads;
    const int slots = (kTc ? ctx->dec_ctas_per_sm : 2) * ctx->sm_count;
    const double row_bytes = 2.0 * kHeadDim * sizeof(KVT);
    constexpr double kRate = 22.6e3;  // bytes per us per CTA
    constexpr double kFixed = 4.0, kMergeCost = 2.0;
    long long chunk = 0;
    double best = 1e300;
    for (int s = 1; s <= kMaxSplit; ++s) {
        long long c = (maxrows + s - 1) / s;
        c = std::max<long long>(c, kMinTiles * TK);
        c = (c + TK - 1) / TK * TK;
        const long long ns = (maxrows + c - 1) / c;
        if (ns > kMaxSplit) continue;
        // short ranges run the fused form, whose last split merges every
        // partial of its (sequence, head) alone: 64 partials measured slower
        // than 32 twice as long (B=1 x 8192 rows: 22.9 vs 18.9 us)
        if (kTc && c < 2048 && ns > 32) continue;
        const long long last = maxrows - (ns - 1) * c;
        const long long big = (long long)units * (ns - (ns > 1 && 4 * last < c ? 1 : 0));
        const long long waves = std::max<long long>(1, (big + slots - 1) / slots);
        const double t = waves * (c * row_bytes / kRate + kFixed + (ns > 1 ? kMergeCost : 0.0));
        if (t < best * (1.0 - 1e-9)) {
            best = t;
            chunk = c;
        }
        if (c == kMinTiles * TK) break;  // smaller splits only repeat this one
    }
    pl.chunk = (int)chunk;
    pl.nsplit = std::max(1, (int)((maxrows + chunk - 1) / chunk));
}

// Runs the split-KV kernel (with the q/k/v prologue fused in).  partial_out
// null: final output into out, the last split of each (seq, kv head)
// merging the partials in the same launch; otherwise one merged (m, l, O)
// partial per (seq, head) into `partial_out` [B][8][258] via merge_partials.
template <typename KVT>
static int decode_impl(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids, const int *pos, const float *Q,
                       const float *K, const float *V, float *out, float *partial_out,
                       const g3::PeerXchg *px = nullptr) {
    DecodePlan pl;
    plan_decode<KVT>(ctx, layer, B, seq_ids, pos, pl);
    g3::LayerDev L = layer_dev(ctx, layer);
    // Long key ranges per CTA (>= 2048 rows): a separate prologue kernel
    // prepares q and appends k/v, so no CTA of the long streaming kernel
    // waits on that work (measured: the fused form cost ~3.5% at B=64 x 32K
    // keys).  Short ranges fold it into the split kernel, saving a launch.
    const bool fused = pl.chunk < 2048;
    g3::DecodeParams p;
    if (!fused) {
        launch_pdl(g3::prologue_decode<KVT>, dim3(B), dim3(512), 0, ctx->stream, Q, K, V, L, ctx->cfg.rmsnorm_eps,
                   pl.rows, ctx->qdec);
        if (int r = check_launch(ctx, 1)) return r;
    }
    p.q = fused ? nullptr : ctx->qdec;
    p.qraw = fused ? Q : nullptr;
    p.kraw = K;
    p.vraw = V;
    p.eps = ctx->cfg.rmsnorm_eps;
    // In-kernel merge (last split merges) for the short fused calls, where a
    // second launch is a large share of the call; long calls keep the
    // separate merge kernel, which measured faster on them.
    p.tickets = (partial_out || !fused) ? nullptr : ctx->tickets;
    p.L = L;
    p.chunk = pl.chunk;
    p.nsplit = pl.nsplit;
    p.partial = ctx->partial;
    p.out = out;
    p.write_partial = (pl.nsplit > 1 || partial_out) ? 1 : 0;
    p.err = ctx->err;
    const int smem = g3::DecodeCfg<KVT>::NS * 2 * g3::DecodeCfg<KVT>::TK * kHeadDim * sizeof(KVT) +
                     (fused ? g3::kFusedExtra<KVT> : 0);
    size_t e0;
    prof_begin(ctx, &e0);
    const dim3 grid(pl.nsplit, kKvHeads, B);
    if constexpr (std::is_same<KVT, __nv_bfloat16>::value) {
        // BF16 cache: both contractions on the tensor core
        const CUtensorMap &tm = ctx->layers[layer].tm_kv;
        if (B <= g3::kSmallDecodeBatch) {
            g3::DecodeRowsSmall rs;
            rs.B = B;
            for (int b = 0; b < B; ++b) {
                rs.seq[b] = pl.rows.seq[b];
                rs.nrows[b] = pl.rows.nrows[b];
                rs.pos[b] = pl.rows.pos[b];
            }
            if (fused)
                launch_pdl(g3::decode_tc<true, g3::DecodeRowsSmall>, grid, dim3(g3::kTcThreads), g3::kTcSmem,
                           ctx->stream, tm, p, rs);
            else
                launch_pdl(g3::decode_tc<false, g3::DecodeRowsSmall>, grid, dim3(g3::kTcThreads), g3::kTcSmem,
                           ctx->stream, tm, p, rs);
        } else if (fused) {
            launch_pdl(g3::decode_tc<true>, grid, dim3(g3::kTcThreads), g3::kTcSmem, ctx->stream, tm, p, pl.rows);
        } else {
            launch_pdl(g3::decode_tc<false>, grid, dim3(g3::kTcThreads), g3::kTcSmem, ctx->stream, tm, p, pl.rows);
        }
    } else if (fused) {
        launch_pdl(g3::decode_splitkv<KVT, true>, grid, dim3(256), smem, ctx->stream, p, pl.rows);
    } else {
        launch_pdl(g3::decode_splitkv<KVT, false>, grid, dim3(256), smem, ctx->stream, p, pl.rows);
    }
    if (ctx->prof) {
        // algorithmic bytes: every attended K and V row once
        double rows = 0;
        for (int b = 0; b < B; ++b) rows += pl.rows.nrows[b];
        prof_end(ctx, 0, e0, rows * kKvHeads * 2.0 * kHeadDim * sizeof(KVT));
    }
    if (int r = check_launch(ctx, 1)) return r;
    if (px) {
        // merged partial straight into every rank's receive buffer (NVLink)
        const size_t hs = (size_t)pl.nsplit * kPartialStride;
        launch_pdl(g3::merge_partials_push, dim3(B * kHeads), dim3(256), 0, ctx->stream, (const float *)ctx->partial,
                   pl.nsplit, (size_t)(kHeads * hs), hs, (size_t)kPartialStride, *px);
        if (int r = check_launch(ctx, 1)) return r;
    } else if (p.write_partial && !p.tickets) {
        const size_t hs = (size_t)pl.nsplit * kPartialStride;
        launch_pdl(g3::merge_partials, dim3(B * kHeads), dim3(256), 0, ctx->stream, (const float *)ctx->partial,
                   pl.nsplit, (size_t)(kHeads * hs), hs, (size_t)kPartialStride, out, partial_out);
        if (int r = check_launch(ctx, 1)) return r;
    }
    return 0;
}

static int decode_dispatch(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids, const int *pos,
                           const float *Q, const float *K, const float *V, float *out, float *partial_out,
                           const g3::PeerXchg *px = nullptr) {
    if (ctx->cfg.kv_dtype == GEMMA3_CUDA_KV_BF16)
        return decode_impl<__nv_bfloat16>(ctx, layer, B, seq_ids, pos, Q, K, V, out, partial_out, px);
    return decode_impl<float>(ctx, layer, B, seq_ids, pos, Q, K, V, out, partial_out, px);
}

// Epoch of the exchange after `e`.  Its parity selects the receive slot and
// must alternate from one exchange to the next; 0 is the flags' initial value,
// so the wrap goes from 0xFFFFFFFF (odd) to 2 (even).
static unsigned next_epoch(unsigned e) { return e == 0xFFFFFFFFu ? 2u : e + 1u; }

// Kernel parameters of the next peer-memory exchange.  The caller advances
// the context's epoch only once the push (which raises the flags) has been
// enqueued, so a launch refused before it leaves the epochs of all ranks in
// step; gemma3_cuda_reset on every rank clears epochs and flags together.
static void peer_params(gemma3_cuda_ctx *ctx, g3::PeerXchg *px) {
    const int R = ctx->cfg.kv_ranks;
    for (int r = 0; r < g3::kMaxPeers; ++r) {
        px->gather[r] = r < R ? ctx->peer_g[r] : nullptr;
        px->flags[r] = r < R ? ctx->peer_f[r] : nullptr;
    }
    px->counter = ctx->pcounter;
    px->rank_stride = (size_t)ctx->cfg.max_batch * kHeads * kPartialStride;
    px->parity_stride = (size_t)R * px->rank_stride;
    px->epoch = next_epoch(ctx->xepoch);
    px->me = ctx->cfg.kv_rank;
    px->R = R;
}

extern "C" int gemma3_cuda_merge_partials_dev(gemma3_cuda_ctx *ctx, int n_parts, int B, const float *partials,
                                              float *out) {
    if (!ctx || n_parts <= 0 || B <= 0 || !partials || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad argument");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    // partials [n_parts][B][8][258]
    g3::merge_partials<<<B * kHeads, 256, 0, ctx->stream>>>(partials, n_parts, (size_t)kHeads * kPartialStride,
                                                             kPartialStride, (size_t)B * kHeads * kPartialStride,
                                                             out, nullptr);
    return check_launch(ctx, 1);
}

extern "C" int gemma3_cuda_attn_decode_partial_dev(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids,
                                                   const int *pos, const float *Q, const float *K, const float *V,
                                                   float *partial) {
    if (int r = decode_check(ctx, layer, B, seq_ids, pos)) return r;
    if (!Q || !K || !V || !partial) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    return decode_dispatch(ctx, layer, B, seq_ids, pos, Q, K, V, nullptr, partial);
}

extern "C" int gemma3_cuda_attn_decode_dev(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids,
                                           const int *pos, const float *Q, const float *K, const float *V,
                                           float *out) {
    if (int r = decode_check(ctx, layer, B, seq_ids, pos)) return r;
    if (!Q || !K || !V || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    const bool split = ctx->layers[layer].is_global && ctx->cfg.kv_ranks > 1;
    if (!split) return decode_dispatch(ctx, layer, B, seq_ids, pos, Q, K, V, out, nullptr);
    if (ctx->use_peer) {
        // fused exchange: merge + NVLink push in one kernel, bounded flag
        // wait + final merge in the next
        g3::PeerXchg px;
        peer_params(ctx, &px);
        if (int r = decode_dispatch(ctx, layer, B, seq_ids, pos, Q, K, V, nullptr, ctx->emit, &px)) return r;
        ctx->xepoch = px.epoch;  // the push is enqueued: it raises this epoch's flags
        launch_pdl(g3::merge_peer_partials, dim3(B * kHeads), dim3(256), 0, ctx->stream, px, out, ctx->err);
        return check_launch(ctx, 1);
    }
    if (!ctx->comm)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG,
                    "global layer of a context-parallel context needs gemma3_cuda_comm_init (or the partial API)");
    if (int r = decode_dispatch(ctx, layer, B, seq_ids, pos, Q, K, V, nullptr, ctx->emit)) return r;
    const size_t n = (size_t)B * kHeads * kPartialStride;
    int nr = g_nccl.allGather(ctx->emit, ctx->gather, n, kNcclFloat32, ctx->comm, ctx->stream);
    if (nr != 0)
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "ncclAllGather failed: %s",
                    g_nccl.getErrorString ? g_nccl.getErrorString(nr) : "?");
    return gemma3_cuda_merge_partials_dev(ctx, ctx->cfg.kv_ranks, B, ctx->gather, out);
}

// Device address of a page-locked (cudaHostAlloc / cudaHostRegister) host
// buffer, or null for ordinary pageable memory.
static const void *mapped_host(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // pageable memory on older runtimes reports an error: clear it
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

extern "C" int gemma3_cuda_attn_decode(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids, const int *pos,
                                       const float *Q, const float *K, const float *V, float *out) {
    if (int r = decode_check(ctx, layer, B, seq_ids, pos)) return r;
    if (!Q || !K || !V || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    float *dq = ctx->io, *dk = dq + (size_t)B * 2048, *dv = dk + (size_t)B * 1024, *dout = dv + (size_t)B * 1024;
    // Page-locked host buffers are used in place: the kernels read q/k/v and
    // write the output across PCIe themselves (inside the launches, so the
    // transfer overlaps the cache streaming), instead of separate copies
    // around them.  When the fused kernel runs several splits per (sequence,
    // kv head), each split reads its q heads itself; that still measured
    // faster than three staging copies (B = 1..16 on a local layer: 29.7 vs
    // 36.2 us ... 43.0 vs 51.7 us per call).  Pageable buffers and
    // context-parallel global layers go through the staging copies.
    const bool split = ctx->layers[layer].is_global && ctx->cfg.kv_ranks > 1;
    const float *hq = nullptr, *hk = nullptr, *hv = nullptr;
    float *hout = nullptr;
    if (!split) {
        hout = (float *)mapped_host(out);
        if (hout) {
            hq = (const float *)mapped_host(Q);
            hk = (const float *)mapped_host(K);
            hv = (const float *)mapped_host(V);
        }
    }
    const bool in_place = hq && hk && hv;
    if (!in_place) {
        CU_TRY(cudaMemcpyAsync(dq, Q, (size_t)B * 2048 * 4, cudaMemcpyHostToDevice, ctx->stream));
        CU_TRY(cudaMemcpyAsync(dk, K, (size_t)B * 1024 * 4, cudaMemcpyHostToDevice, ctx->stream));
        CU_TRY(cudaMemcpyAsync(dv, V, (size_t)B * 1024 * 4, cudaMemcpyHostToDevice, ctx->stream));
    }
    if (int r = gemma3_cuda_attn_decode_dev(ctx, layer, B, seq_ids, pos, in_place ? hq : dq, in_place ? hk : dk,
                                            in_place ? hv : dv, hout ? hout : dout))
        return r;
    if (!hout) CU_TRY(cudaMemcpyAsync(out, dout, (size_t)B * 2048 * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return gemma3_cuda_synchronize(ctx);
}

// ------------------------------------------------------------------ projections
// Q/K/V and O projections of layer_attention (gemma3_transformer.c:290-292,
// :355) and of the batched prefill (:614-639, :694-699) on the tensor cores:
// BF16 weights resident in HBM, the activations rounded to BF16 once, fp32
// accumulation (kernels in proj_kernels.cuh).
static constexpr int kHidden = 2560;
static constexpr int kQSize = kHeads * kHeadDim;     // 2048
static constexpr int kKvSize = kKvHeads * kHeadDim;  // 1024
static constexpr int kQkvRows = kQSize + 2 * kKvSize;

static int proj_scratch(gemma3_cuda_ctx *c, int rows) {
    if (c->proj_rows >= rows) return 0;
    cudaFree(c->xb);
    cudaFree(c->ab);
    cudaFree(c->qkv);
    cudaFree(c->attn);
    cudaFree(c->xio);
    c->xb = c->ab = nullptr;
    c->qkv = c->attn = c->xio = nullptr;
    c->proj_rows = 0;
    CU_TRY(cudaMalloc(&c->xb, (size_t)rows * kHidden * 2));
    CU_TRY(cudaMalloc(&c->ab, (size_t)rows * kQSize * 2));
    CU_TRY(cudaMalloc(&c->qkv, (size_t)rows * kQkvRows * 4));
    CU_TRY(cudaMalloc(&c->attn, (size_t)rows * kQSize * 4));
    CU_TRY(cudaMalloc(&c->xio, (size_t)rows * kHidden * 4 * 2));
    c->proj_rows = rows;
    return 0;
}

// fp16 matrix [rows][cols] (row-major), box 64 columns x box_rows rows, 128-byte swizzle.
static int make_map_f16(CUtensorMap *m, const void *base, int rows, int cols, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

// Y[T][N] = X[T][K] . W[N][K]^T, routed by `out`.  xb: fp16 [T][K] (device).
// deferred: null, or where a caller that sums the split-K partials itself
// (residual_norm_rows) gets their count: 0 = the output is in `out` (one
// split), S > 1 = S partial sums [S][T][N] in ctx->pp, no reduce launched.
static int proj_run(gemma3_cuda_ctx *ctx, const __half *W, int N, int K, const __half *xb, int T,
                    const g3::ProjOut &out, int *deferred = nullptr) {
    const int nt = std::min(256, (T + 31) / 32 * 32);  // the epilogue reads 32 tokens per tcgen05.ld
    const int ntile_tok = (T + nt - 1) / nt;
    const int mtiles = N / 128, kchunks = K / 64;
    const int tiles = mtiles * ntile_tok;
    // Too few tiles to keep every SM busy (decode): split K.  The split count
    // minimises the busiest SM's work in 64-wide K chunks, (tiles per SM) x
    // (chunks per tile + 2 for writing and reducing a tile's partial sums),
    // preferring fewer splits on ties; no split is empty.
    int splits = 1;
    if (tiles < ctx->sm_count) {
        long best = kchunks;  // one split: every tile does all chunks
        for (int sp = 2; sp <= kchunks; ++sp) {
            const int kper = (kchunks + sp - 1) / sp;
            const int eff = (kchunks + kper - 1) / kper;
            const long cost = (long)((tiles * eff + ctx->sm_count - 1) / ctx->sm_count) * (kper + 2);
            if (cost < best) {
                best = cost;
                splits = eff;
            }
        }
    }
    if (splits > 1) {
        const size_t need = (size_t)splits * T * N;
        if (ctx->pp_floats < need) {
            cudaFree(ctx->pp);
            ctx->pp = nullptr;
            ctx->pp_floats = 0;
            CU_TRY(cudaMalloc(&ctx->pp, need * 4));
            ctx->pp_floats = need;
        }
    }
    CUtensorMap tw, tx;
    if (int r = make_map_f16(&tw, W, N, K, 128)) return r;
    if (int r = make_map_f16(&tx, xb, T, K, nt)) return r;
    g3::ProjParams p;
    p.T = T;
    p.N = N;
    p.kchunks = kchunks;
    p.nt = nt;
    p.splits = splits;
    p.ntile_tok = ntile_tok;
    p.out = out;
    p.partial = ctx->pp;
    p.err = ctx->err;
    const int grid = std::min(tiles * splits, ctx->sm_count);
    size_t e0;
    prof_begin(ctx, &e0);
    CU_TRY(launch_pdl(g3::proj_gemm_sm100, dim3(grid), dim3(g3::kProjThreads), g3::kProjSmem, ctx->stream, tw, tx, p));
    if (int r = check_launch(ctx, 1)) return r;
    if (deferred) *deferred = splits > 1 ? splits : 0;
    if (splits > 1 && !deferred) {
        const size_t n = (size_t)T * N;
        const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)ctx->sm_count * 8);
        CU_TRY(launch_pdl(g3::proj_splitk_reduce, dim3(blocks), dim3(256), 0, ctx->stream, (const float *)ctx->pp,
                          splits, T, N, out));
        if (int r = check_launch(ctx, 1)) return r;
    }
    prof_end(ctx, 2, e0, 2.0 * T * N * K);
    return 0;
}

static int to_f16(gemma3_cuda_ctx *ctx, const float *x, __half *y, size_t n) {
    const size_t n4 = n / 4;
    const int blocks = (int)std::min<size_t>((n4 + 255) / 256, (size_t)ctx->sm_count * 8);
    CU_TRY(launch_pdl(g3::to_f16_rows, dim3(blocks), dim3(256), 0, ctx->stream, x, y, n4, ctx->err));
    return check_launch(ctx, 1);
}

static int proj_check(gemma3_cuda_ctx *ctx, int layer, int T) {
    if (!ctx || layer < 0 || layer >= ctx->cfg.num_layers) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad layer");
    const int maxT = std::max(ctx->cfg.max_prefill, ctx->cfg.max_batch);
    if (T <= 0 || T > maxT) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad token count %d (max %d)", T, maxT);
    if (!ctx->layers[layer].wqkv) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "projection weights of layer %d not set", layer);
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    return proj_scratch(ctx, maxT);
}

// Host BF16 matrix -> device fp16 (through a staging buffer; the conversion
// runs on the device, see bf16_to_f16).
static int upload_f16(gemma3_cuda_ctx *ctx, __half *dst, const uint16_t *src, size_t n) {
    if (ctx->wstage_elems < n) {
        cudaFree(ctx->wstage);
        ctx->wstage = nullptr;
        ctx->wstage_elems = 0;
        CU_TRY(cudaMalloc(&ctx->wstage, n * 2));
        ctx->wstage_elems = n;
    }
    CU_TRY(cudaMemcpyAsync(ctx->wstage, src, n * 2, cudaMemcpyHostToDevice, ctx->stream));
    const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)ctx->sm_count * 16);
    g3::bf16_to_f16<<<blocks, 256, 0, ctx->stream>>>(ctx->wstage, dst, n, ctx->err);
    return check_launch(ctx, 1);
}

extern "C" int gemma3_cuda_set_proj_weights(gemma3_cuda_ctx *ctx, int layer, const uint16_t *wq, const uint16_t *wk,
                                            const uint16_t *wv, const uint16_t *wo) {
    if (!ctx || layer < 0 || layer >= ctx->cfg.num_layers) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad layer");
    if (!wq || !wk || !wv || !wo) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null weight");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    LayerState &L = ctx->layers[layer];
    if (!L.wqkv) CU_TRY(cudaMalloc(&L.wqkv, (size_t)kQkvRows * kHidden * 2));
    if (!L.wo) CU_TRY(cudaMalloc(&L.wo, (size_t)kHidden * kQSize * 2));
    if (int r = upload_f16(ctx, L.wqkv, wq, (size_t)kQSize * kHidden)) return r;
    if (int r = upload_f16(ctx, L.wqkv + (size_t)kQSize * kHidden, wk, (size_t)kKvSize * kHidden)) return r;
    if (int r = upload_f16(ctx, L.wqkv + (size_t)(kQSize + kKvSize) * kHidden, wv, (size_t)kKvSize * kHidden))
        return r;
    if (int r = upload_f16(ctx, L.wo, wo, (size_t)kHidden * kQSize)) return r;
    return gemma3_cuda_synchronize(ctx);  // a weight outside the fp16 range fails here
}

extern "C" int gemma3_cuda_project_qkv_dev(gemma3_cuda_ctx *ctx, int layer, int T, const float *x, float *q, float *k,
                                           float *v) {
    if (int r = proj_check(ctx, layer, T)) return r;
    if (!x || !q || !k || !v) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    if (int r = to_f16(ctx, x, ctx->xb, (size_t)T * kHidden)) return r;
    g3::ProjOut o;
    o.ptr[0] = q;
    o.ptr[1] = k;
    o.ptr[2] = v;
    o.ld[0] = kQSize;
    o.ld[1] = o.ld[2] = kKvSize;
    o.lo[0] = 0;
    o.lo[1] = kQSize;
    o.lo[2] = kQSize + kKvSize;
    o.lo[3] = kQkvRows;
    return proj_run(ctx, ctx->layers[layer].wqkv, kQkvRows, kHidden, ctx->xb, T, o);
}

extern "C" int gemma3_cuda_project_o_dev(gemma3_cuda_ctx *ctx, int layer, int T, const float *attn, float *out) {
    if (int r = proj_check(ctx, layer, T)) return r;
    if (!attn || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    if (int r = to_f16(ctx, attn, ctx->ab, (size_t)T * kQSize)) return r;
    g3::ProjOut o;
    o.ptr[0] = o.ptr[1] = o.ptr[2] = out;
    o.ld[0] = o.ld[1] = o.ld[2] = kHidden;
    o.lo[0] = 0;
    o.lo[1] = o.lo[2] = o.lo[3] = kHidden;
    return proj_run(ctx, ctx->layers[layer].wo, kHidden, kQSize, ctx->ab, T, o);
}

extern "C" int gemma3_cuda_layer_decode_dev(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids,
                                            const int *pos, const float *x, float *out) {
    if (int r = proj_check(ctx, layer, B)) return r;
    float *q = ctx->qkv, *k = q + (size_t)ctx->proj_rows * kQSize, *v = k + (size_t)ctx->proj_rows * kKvSize;
    if (int r = gemma3_cuda_project_qkv_dev(ctx, layer, B, x, q, k, v)) return r;
    if (int r = gemma3_cuda_attn_decode_dev(ctx, layer, B, seq_ids, pos, q, k, v, ctx->attn)) return r;
    return gemma3_cuda_project_o_dev(ctx, layer, B, ctx->attn, out);
}

extern "C" int gemma3_cuda_layer_decode(gemma3_cuda_ctx *ctx, int layer, int B, const int *seq_ids, const int *pos,
                                        const float *x, float *out) {
    if (int r = proj_check(ctx, layer, B)) return r;
    if (!x || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    float *dx = ctx->xio, *dout = dx + (size_t)ctx->proj_rows * kHidden;
    CU_TRY(cudaMemcpyAsync(dx, x, (size_t)B * kHidden * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (int r = gemma3_cuda_layer_decode_dev(ctx, layer, B, seq_ids, pos, dx, dout)) return r;
    CU_TRY(cudaMemcpyAsync(out, dout, (size_t)B * kHidden * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return gemma3_cuda_synchronize(ctx);
}

extern "C" int gemma3_cuda_layer_prefill_dev(gemma3_cuda_ctx *ctx, int layer, int seq, const float *x, int T,
                                             int start_pos, float *out) {
    if (int r = proj_check(ctx, layer, T)) return r;
    float *q = ctx->qkv, *k = q + (size_t)ctx->proj_rows * kQSize, *v = k + (size_t)ctx->proj_rows * kKvSize;
    if (int r = gemma3_cuda_project_qkv_dev(ctx, layer, T, x, q, k, v)) return r;
    if (int r = gemma3_cuda_attn_prefill_dev(ctx, layer, seq, q, k, v, T, start_pos, ctx->attn)) return r;
    return gemma3_cuda_project_o_dev(ctx, layer, T, ctx->attn, out);
}

extern "C" int gemma3_cuda_layer_prefill(gemma3_cuda_ctx *ctx, int layer, int seq, const float *x, int T,
                                         int start_pos, float *out) {
    if (int r = proj_check(ctx, layer, T)) return r;
    if (!x || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    float *dx = ctx->xio, *dout = dx + (size_t)ctx->proj_rows * kHidden;
    CU_TRY(cudaMemcpyAsync(dx, x, (size_t)T * kHidden * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (int r = gemma3_cuda_layer_prefill_dev(ctx, layer, seq, dx, T, start_pos, dout)) return r;
    CU_TRY(cudaMemcpyAsync(out, dout, (size_t)T * kHidden * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return gemma3_cuda_synchronize(ctx);
}

// ------------------------------------------------------------------ transformer block
// The whole Gemma 3 block on the device (gemma3_transformer_forward,
// gemma3_transformer.c:427-499): input norm, attention (projections
// included), post-attention norm + residual, pre-FFN norm, gated GELU MLP
// (layer_mlp, :362-398), post-FFN norm + residual; the residual stream stays
// in device memory across all layers.
static constexpr int kInter = 10240;  // intermediate_size of Gemma 3 4B

static int block_scratch(gemma3_cuda_ctx *c, int rows) {
    if (c->blk_rows >= rows) return 0;
    cudaFree(c->gu);
    cudaFree(c->hb);
    cudaFree(c->delta);
    cudaFree(c->xfwd);
    c->gu = nullptr;
    c->hb = nullptr;
    c->delta = c->xfwd = nullptr;
    c->blk_rows = 0;
    CU_TRY(cudaMalloc(&c->gu, (size_t)rows * 2 * kInter * 4));
    CU_TRY(cudaMalloc(&c->hb, (size_t)rows * kInter * 2));
    CU_TRY(cudaMalloc(&c->delta, (size_t)rows * kHidden * 4));
    CU_TRY(cudaMalloc(&c->xfwd, (size_t)rows * kHidden * 4));
    c->blk_rows = rows;
    return 0;
}

extern "C" int gemma3_cuda_set_layer_weights(gemma3_cuda_ctx *ctx, int layer, const gemma3_cuda_layer_weights *w) {
    if (!ctx || !w || layer < 0 || layer >= ctx->cfg.num_layers) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad layer");
    if (!w->gate_proj || !w->up_proj || !w->down_proj || !w->input_layernorm)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null weight");
    if (int r = gemma3_cuda_set_proj_weights(ctx, layer, w->q_proj, w->k_proj, w->v_proj, w->o_proj)) return r;
    if (int r = gemma3_cuda_set_qk_norm(ctx, layer, w->q_norm, w->k_norm)) return r;
    LayerState &L = ctx->layers[layer];
    L.block_ready = 0;
    if (!L.wgu) CU_TRY(cudaMalloc(&L.wgu, (size_t)2 * kInter * kHidden * 2));
    if (!L.wdown) CU_TRY(cudaMalloc(&L.wdown, (size_t)kHidden * kInter * 2));
    if (!L.ln) CU_TRY(cudaMalloc(&L.ln, (size_t)4 * kHidden * 2));
    if (int r = upload_f16(ctx, L.wgu, w->gate_proj, (size_t)kInter * kHidden)) return r;
    if (int r = upload_f16(ctx, L.wgu + (size_t)kInter * kHidden, w->up_proj, (size_t)kInter * kHidden)) return r;
    if (int r = upload_f16(ctx, L.wdown, w->down_proj, (size_t)kHidden * kInter)) return r;
    const uint16_t *lns[4] = {w->input_layernorm, w->post_attention_layernorm, w->pre_feedforward_layernorm,
                              w->post_feedforward_layernorm};
    for (int i = 0; i < 4; ++i) {
        L.ln_set[i] = lns[i] ? 1 : 0;  // a missing post / pre-FFN norm is skipped, as the reference does
        if (lns[i])
            CU_TRY(cudaMemcpyAsync(L.ln + (size_t)i * kHidden, lns[i], kHidden * 2, cudaMemcpyHostToDevice,
                                   ctx->stream));
    }
    if (int r = gemma3_cuda_synchronize(ctx)) return r;
    L.block_ready = 1;
    return 0;
}

static const uint16_t *ln_of(const LayerState &L, int i) { return L.ln_set[i] ? L.ln + (size_t)i * kHidden : nullptr; }

// x [T][2560] (device, fp32) <- all layers applied to T rows.  attn(l, q, k,
// v, out) runs the attention core of layer l on the rows.
template <typename AttnFn>
static int forward_layers(gemma3_cuda_ctx *ctx, int T, float *x, AttnFn attn) {
    for (int l = 0; l < ctx->cfg.num_layers; ++l)
        if (!ctx->layers[l].block_ready)
            return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "block weights of layer %d not set", l);
    if (int r = proj_check(ctx, 0, T)) return r;
    if (int r = block_scratch(ctx, ctx->proj_rows)) return r;
    const float eps = ctx->cfg.rmsnorm_eps;
    const int R = ctx->proj_rows;
    float *q = ctx->qkv, *k = q + (size_t)R * kQSize, *v = k + (size_t)R * kKvSize;
    float *gate = ctx->gu, *up = ctx->gu + (size_t)R * kInter;
    // pre-attention norm of layer 0; every later one comes out of the
    // previous layer's last residual step
    CU_TRY(launch_pdl(g3::rms_norm_rows_f16, dim3(T), dim3(g3::kNormThreads), 0, ctx->stream, (const float *)x,
                      ln_of(ctx->layers[0], 0), ctx->xb, eps, ctx->err));
    if (int r = check_launch(ctx, 1)) return r;
    for (int l = 0; l < ctx->cfg.num_layers; ++l) {
        const LayerState &L = ctx->layers[l];
        g3::ProjOut o;
        o.ptr[0] = q;
        o.ptr[1] = k;
        o.ptr[2] = v;
        o.ld[0] = kQSize;
        o.ld[1] = o.ld[2] = kKvSize;
        o.lo[0] = 0;
        o.lo[1] = kQSize;
        o.lo[2] = kQSize + kKvSize;
        o.lo[3] = kQkvRows;
        if (int r = proj_run(ctx, L.wqkv, kQkvRows, kHidden, ctx->xb, T, o)) return r;
        if (int r = attn(l, q, k, v, ctx->attn)) return r;
        if (int r = to_f16(ctx, ctx->attn, ctx->ab, (size_t)T * kQSize)) return r;
        o.ptr[0] = o.ptr[1] = o.ptr[2] = ctx->delta;
        o.ld[0] = o.ld[1] = o.ld[2] = kHidden;
        o.lo[0] = 0;
        o.lo[1] = o.lo[2] = o.lo[3] = kHidden;
        // the split-K partials of O and down are summed by residual_norm_rows
        // (in split order, as the reduce kernel would), one launch fewer each
        int ds = 0;
        if (int r = proj_run(ctx, L.wo, kHidden, kQSize, ctx->ab, T, o, &ds)) return r;
        // x += post_attn_norm(o_proj); xn = pre_ffn_norm(x)
        CU_TRY(launch_pdl(g3::residual_norm_rows, dim3(T), dim3(g3::kNormThreads), 0, ctx->stream,
                          (const float *)(ds ? ctx->pp : ctx->delta), ds ? ds : 1, (size_t)T * kHidden, ln_of(L, 1),
                          x, ln_of(L, 2), ctx->xb, eps, ctx->err));
        if (int r = check_launch(ctx, 1)) return r;
        o.ptr[0] = gate;
        o.ptr[1] = o.ptr[2] = up;
        o.ld[0] = o.ld[1] = o.ld[2] = kInter;
        o.lo[0] = 0;
        o.lo[1] = o.lo[2] = kInter;
        o.lo[3] = 2 * kInter;
        if (int r = proj_run(ctx, L.wgu, 2 * kInter, kHidden, ctx->xb, T, o)) return r;
        {
            const size_t n = (size_t)T * kInter;
            // gate and up rows are [T][10240] each, contiguous
            const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)ctx->sm_count * 8);
            CU_TRY(launch_pdl(g3::gelu_mul_f16, dim3(blocks), dim3(256), 0, ctx->stream, (const float *)gate,
                              (const float *)up, ctx->hb, n, ctx->err));
            if (int r = check_launch(ctx, 1)) return r;
        }
        o.ptr[0] = o.ptr[1] = o.ptr[2] = ctx->delta;
        o.ld[0] = o.ld[1] = o.ld[2] = kHidden;
        o.lo[0] = 0;
        o.lo[1] = o.lo[2] = o.lo[3] = kHidden;
        if (int r = proj_run(ctx, L.wdown, kHidden, kInter, ctx->hb, T, o, &ds)) return r;
        // x += post_ffn_norm(mlp); xn = next layer's pre-attention norm(x)
        const bool last = l + 1 == ctx->cfg.num_layers;
        CU_TRY(launch_pdl(g3::residual_norm_rows, dim3(T), dim3(g3::kNormThreads), 0, ctx->stream,
                          (const float *)(ds ? ctx->pp : ctx->delta), ds ? ds : 1, (size_t)T * kHidden, ln_of(L, 3), x,
                          last ? (const uint16_t *)nullptr : ln_of(ctx->layers[l + 1], 0),
                          last ? (__half *)nullptr : ctx->xb, eps, ctx->err));
        if (int r = check_launch(ctx, 1)) return r;
    }
    return 0;
}

extern "C" int gemma3_cuda_forward_dev(gemma3_cuda_ctx *ctx, int B, const int *seq_ids, const int *pos, float *x) {
    if (int r = decode_check(ctx, 0, B, seq_ids, pos)) return r;
    if (!x) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    return forward_layers(ctx, B, x, [&](int l, const float *q, const float *k, const float *v, float *out) {
        return gemma3_cuda_attn_decode_dev(ctx, l, B, seq_ids, pos, q, k, v, out);
    });
}

extern "C" int gemma3_cuda_forward(gemma3_cuda_ctx *ctx, int B, const int *seq_ids, const int *pos, float *x) {
    if (int r = decode_check(ctx, 0, B, seq_ids, pos)) return r;
    if (!x) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    if (int r = proj_check(ctx, 0, B)) return r;
    if (int r = block_scratch(ctx, ctx->proj_rows)) return r;
    CU_TRY(cudaMemcpyAsync(ctx->xfwd, x, (size_t)B * kHidden * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (int r = gemma3_cuda_forward_dev(ctx, B, seq_ids, pos, ctx->xfwd)) return r;
    CU_TRY(cudaMemcpyAsync(x, ctx->xfwd, (size_t)B * kHidden * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return gemma3_cuda_synchronize(ctx);
}

extern "C" int gemma3_cuda_prefill_forward_dev(gemma3_cuda_ctx *ctx, int seq, float *x, int T, int start_pos) {
    for (int l = 0; l < ctx->cfg.num_layers; ++l)
        if (int r = prefill_check(ctx, l, seq, T, start_pos)) return r;
    if (!x) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    return forward_layers(ctx, T, x, [&](int l, const float *q, const float *k, const float *v, float *out) {
        return gemma3_cuda_attn_prefill_dev(ctx, l, seq, q, k, v, T, start_pos, out);
    });
}

extern "C" int gemma3_cuda_prefill_forward(gemma3_cuda_ctx *ctx, int seq, float *x, int T, int start_pos) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    if (!x) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    if (int r = proj_check(ctx, 0, T)) return r;
    if (int r = block_scratch(ctx, ctx->proj_rows)) return r;
    CU_TRY(cudaMemcpyAsync(ctx->xfwd, x, (size_t)T * kHidden * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (int r = gemma3_cuda_prefill_forward_dev(ctx, seq, ctx->xfwd, T, start_pos)) return r;
    CU_TRY(cudaMemcpyAsync(x, ctx->xfwd, (size_t)T * kHidden * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return gemma3_cuda_synchronize(ctx);
}

// ------------------------------------------------------------------ greedy decoding
// Embedding lookup (gemma3_embed_bf16 + the sqrt(hidden) scale), the 34
// blocks, the final norm and the tied-embedding logits (gemma3_transformer.c:
// 502-509) with the greedy argmax (gemma3_argmax) on the device.
extern "C" int gemma3_cuda_set_embeddings(gemma3_cuda_ctx *ctx, const uint16_t *embed, int vocab,
                                          const uint16_t *final_norm) {
    if (!ctx || !embed || !final_norm || vocab <= 0) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad embedding arguments");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    cudaFree(ctx->embed);
    cudaFree(ctx->embed16);
    cudaFree(ctx->logits);
    ctx->embed = nullptr;
    ctx->embed16 = nullptr;
    ctx->logits = nullptr;
    ctx->logit_rows = 0;
    ctx->vocab = ctx->vocab_pad = 0;
    const int pad = (vocab + 127) / 128 * 128;
    CU_TRY(cudaMalloc(&ctx->embed, (size_t)vocab * kHidden * 2));
    CU_TRY(cudaMalloc(&ctx->embed16, (size_t)pad * kHidden * 2));
    if (!ctx->final_ln) CU_TRY(cudaMalloc(&ctx->final_ln, kHidden * 2));
    CU_TRY(cudaMemcpyAsync(ctx->embed, embed, (size_t)vocab * kHidden * 2, cudaMemcpyHostToDevice, ctx->stream));
    CU_TRY(cudaMemcpyAsync(ctx->final_ln, final_norm, kHidden * 2, cudaMemcpyHostToDevice, ctx->stream));
    CU_TRY(cudaMemsetAsync(ctx->embed16 + (size_t)vocab * kHidden, 0, (size_t)(pad - vocab) * kHidden * 2, ctx->stream));
    {
        const size_t n = (size_t)vocab * kHidden;
        const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)ctx->sm_count * 16);
        g3::bf16_to_f16<<<blocks, 256, 0, ctx->stream>>>(ctx->embed, ctx->embed16, n, ctx->err);
        if (int r = check_launch(ctx, 1)) return r;
    }
    if (int r = gemma3_cuda_synchronize(ctx)) return r;
    ctx->vocab = vocab;
    ctx->vocab_pad = pad;
    return 0;
}

// tokens (device [T]) -> x (device [T][2560]) scaled embeddings
static int embed_tokens(gemma3_cuda_ctx *ctx, const int *tokens, int T, float *x) {
    const float scale = sqrtf((float)kHidden);
    CU_TRY(launch_pdl(g3::embed_rows, dim3(T), dim3(g3::kNormThreads), 0, ctx->stream, tokens,
                      (const uint16_t *)ctx->embed, ctx->vocab, scale, x, ctx->err));
    return check_launch(ctx, 1);
}

// rows of x (device [rows][2560]) -> next tokens into ctx->tok_dev, top-1 logits into ctx->top_dev
static int logits_argmax(gemma3_cuda_ctx *ctx, const float *x, int rows) {
    if (ctx->logit_rows < rows) {
        cudaFree(ctx->logits);
        ctx->logits = nullptr;
        ctx->logit_rows = 0;
        CU_TRY(cudaMalloc(&ctx->logits, (size_t)rows * ctx->vocab_pad * 4));
        ctx->logit_rows = rows;
    }
    CU_TRY(launch_pdl(g3::rms_norm_rows_f16, dim3(rows), dim3(g3::kNormThreads), 0, ctx->stream, x,
                      (const uint16_t *)ctx->final_ln, ctx->xb, ctx->cfg.rmsnorm_eps, ctx->err));
    if (int r = check_launch(ctx, 1)) return r;
    g3::ProjOut o;
    o.ptr[0] = o.ptr[1] = o.ptr[2] = ctx->logits;
    o.ld[0] = o.ld[1] = o.ld[2] = ctx->vocab_pad;
    o.lo[0] = 0;
    o.lo[1] = o.lo[2] = o.lo[3] = ctx->vocab_pad;
    if (int r = proj_run(ctx, ctx->embed16, ctx->vocab_pad, kHidden, ctx->xb, rows, o)) return r;
    CU_TRY(launch_pdl(g3::argmax_rows, dim3(rows), dim3(g3::kArgmaxThreads), 0, ctx->stream,
                      (const float *)ctx->logits, (size_t)ctx->vocab_pad, ctx->vocab, ctx->tok_dev, ctx->top_dev));
    return check_launch(ctx, 1);
}

static int greedy_check(gemma3_cuda_ctx *ctx, int rows) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    if (!ctx->vocab) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "embeddings not set");
    if (int r = proj_check(ctx, 0, rows)) return r;
    if (int r = block_scratch(ctx, ctx->proj_rows)) return r;
    if (!ctx->tok_dev) {
        CU_TRY(cudaMalloc(&ctx->tok_dev, (size_t)ctx->proj_rows * 4));
        CU_TRY(cudaMalloc(&ctx->top_dev, (size_t)ctx->proj_rows * 4));
    }
    return 0;
}

extern "C" int gemma3_cuda_prefill_greedy(gemma3_cuda_ctx *ctx, int seq, const int *tokens, int T, int start_pos,
                                          int *next_token, float *top_logit) {
    if (int r = greedy_check(ctx, T)) return r;
    if (!tokens || !next_token) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaMemcpyAsync(ctx->tok_dev, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (int r = embed_tokens(ctx, ctx->tok_dev, T, ctx->xfwd)) return r;
    if (int r = gemma3_cuda_prefill_forward_dev(ctx, seq, ctx->xfwd, T, start_pos)) return r;
    if (int r = logits_argmax(ctx, ctx->xfwd + (size_t)(T - 1) * kHidden, 1)) return r;  // the last prompt token
    CU_TRY(cudaMemcpyAsync(next_token, ctx->tok_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (top_logit) CU_TRY(cudaMemcpyAsync(top_logit, ctx->top_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
    return gemma3_cuda_synchronize(ctx);
}

extern "C" int gemma3_cuda_greedy_step(gemma3_cuda_ctx *ctx, int B, const int *seq_ids, const int *pos,
                                       const int *tokens, int *next_tokens, float *top_logits) {
    if (int r = greedy_check(ctx, B)) return r;
    if (int r = decode_check(ctx, 0, B, seq_ids, pos)) return r;
    if (!tokens || !next_tokens) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaMemcpyAsync(ctx->tok_dev, tokens, (size_t)B * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (int r = embed_tokens(ctx, ctx->tok_dev, B, ctx->xfwd)) return r;
    if (int r = gemma3_cuda_forward_dev(ctx, B, seq_ids, pos, ctx->xfwd)) return r;
    if (int r = logits_argmax(ctx, ctx->xfwd, B)) return r;
    CU_TRY(cudaMemcpyAsync(next_tokens, ctx->tok_dev, (size_t)B * 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (top_logits) CU_TRY(cudaMemcpyAsync(top_logits, ctx->top_dev, (size_t)B * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return gemma3_cuda_synchronize(ctx);
}

// ------------------------------------------------------------------ SafeTensors upload
// The weight names and the BF16 expectation of gemma3_load_weights
// (gemma3_safetensors.c:651-713), checked here (presence, dtype, shape)
// before anything is uploaded; text-only checkpoints without the
// "language_model." prefix are accepted too.
struct StModel {
    std::string prefix;
    std::vector<gemma3_cuda_layer_weights> layers;
    const uint16_t *embed = nullptr, *norm = nullptr;
    int vocab = 0;
};

static std::string shape_str(const std::vector<int64_t> &v) {
    std::string r = "[";
    for (size_t i = 0; i < v.size(); ++i) r += (i ? ", " : "") + std::to_string(v[i]);
    return r + "]";
}

static int st_get(const g3st::Index &ix, const std::string &name, const std::vector<int64_t> &shape, bool required,
                  const uint16_t **out) {
    *out = nullptr;
    const g3st::Tensor *t = ix.find(name);
    if (!t) return required ? fail(GEMMA3_CUDA_ERR_INVALID_ARG, "tensor %s not found", name.c_str()) : 0;
    if (t->dtype != "BF16")
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "tensor %s is %s, not BF16", name.c_str(), t->dtype.c_str());
    if (t->shape != shape)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "tensor %s has shape %s, expected %s", name.c_str(),
                    shape_str(t->shape).c_str(), shape_str(shape).c_str());
    int64_t n = 1;
    for (auto d : shape) n *= d;
    if (t->bytes != (size_t)n * 2)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "tensor %s: %zu bytes for %lld BF16 values", name.c_str(), t->bytes,
                    (long long)n);
    *out = reinterpret_cast<const uint16_t *>(t->data);
    return 0;
}

static int st_collect(const g3st::Index &ix, int num_layers, StModel &m) {
    m.prefix.clear();
    for (const char *pre : {"language_model.model.", "model."})
        if (ix.find(std::string(pre) + "embed_tokens.weight")) {
            m.prefix = pre;
            break;
        }
    if (m.prefix.empty()) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "tensor language_model.model.embed_tokens.weight not found");
    const g3st::Tensor *e = ix.find(m.prefix + "embed_tokens.weight");
    if (e->shape.size() != 2 || e->shape[1] != kHidden || e->shape[0] <= 0 || e->shape[0] > INT32_MAX)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "embed_tokens has shape %s", shape_str(e->shape).c_str());
    m.vocab = (int)e->shape[0];
    if (int r = st_get(ix, m.prefix + "embed_tokens.weight", {m.vocab, kHidden}, true, &m.embed)) return r;
    if (int r = st_get(ix, m.prefix + "norm.weight", {kHidden}, true, &m.norm)) return r;
    m.layers.assign(num_layers, gemma3_cuda_layer_weights{});
    for (int l = 0; l < num_layers; ++l) {
        const std::string p = m.prefix + "layers." + std::to_string(l) + ".";
        gemma3_cuda_layer_weights &w = m.layers[l];
        const struct { const char *name; std::vector<int64_t> shape; bool req; const uint16_t **dst; } items[] = {
            {"input_layernorm.weight", {kHidden}, true, &w.input_layernorm},
            {"self_attn.q_proj.weight", {kQSize, kHidden}, true, &w.q_proj},
            {"self_attn.k_proj.weight", {kKvSize, kHidden}, true, &w.k_proj},
            {"self_attn.v_proj.weight", {kKvSize, kHidden}, true, &w.v_proj},
            {"self_attn.o_proj.weight", {kHidden, kQSize}, true, &w.o_proj},
            {"self_attn.q_norm.weight", {kHeadDim}, false, &w.q_norm},
            {"self_attn.k_norm.weight", {kHeadDim}, false, &w.k_norm},
            {"post_attention_layernorm.weight", {kHidden}, false, &w.post_attention_layernorm},
            {"mlp.gate_proj.weight", {kInter, kHidden}, true, &w.gate_proj},
            {"mlp.up_proj.weight", {kInter, kHidden}, true, &w.up_proj},
            {"mlp.down_proj.weight", {kHidden, kInter}, true, &w.down_proj},
            {"pre_feedforward_layernorm.weight", {kHidden}, false, &w.pre_feedforward_layernorm},
            {"post_feedforward_layernorm.weight", {kHidden}, false, &w.post_feedforward_layernorm},
        };
        for (const auto &it : items)
            if (int r = st_get(ix, p + it.name, it.shape, it.req, it.dst)) return r;
    }
    return 0;
}

extern "C" int gemma3_cuda_safetensors_check(const char *model_dir, int num_layers, int *vocab_out) {
    if (!model_dir || num_layers <= 0) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad arguments");
    g3st::Index ix;
    std::string err;
    if (!ix.open(model_dir, err)) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "%s", err.c_str());
    StModel m;
    if (int r = st_collect(ix, num_layers, m)) return r;
    if (vocab_out) *vocab_out = m.vocab;
    return 0;
}

extern "C" int gemma3_cuda_load_safetensors(gemma3_cuda_ctx *ctx, const char *model_dir) {
    if (!ctx || !model_dir) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad arguments");
    g3st::Index ix;
    std::string err;
    if (!ix.open(model_dir, err)) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "%s", err.c_str());
    StModel m;
    if (int r = st_collect(ix, ctx->cfg.num_layers, m)) return r;  // everything checked before any upload
    for (int l = 0; l < ctx->cfg.num_layers; ++l)
        if (int r = gemma3_cuda_set_layer_weights(ctx, l, &m.layers[l])) return r;
    return gemma3_cuda_set_embeddings(ctx, m.embed, m.vocab, m.norm);
}

// ------------------------------------------------------------------ NCCL
extern "C" int gemma3_cuda_comm_unique_id(void *id_128_bytes) {
    if (!id_128_bytes) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null id buffer");
    if (int r = nccl_load()) return r;
    g3NcclUniqueId id;
    int nr = g_nccl.getUniqueId(&id);
    if (nr != 0) return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "ncclGetUniqueId failed (%d)", nr);
    memcpy(id_128_bytes, id.internal, 128);
    return 0;
}

extern "C" int gemma3_cuda_comm_init(gemma3_cuda_ctx *ctx, const void *id_128_bytes) {
    if (!ctx || !id_128_bytes) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null argument");
    if (int r = nccl_load()) return r;
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    g3NcclUniqueId id;
    memcpy(id.internal, id_128_bytes, 128);
    int nr = g_nccl.commInitRank(&ctx->comm, ctx->cfg.kv_ranks, id, ctx->cfg.kv_rank);
    if (nr != 0) {
        ctx->comm = nullptr;
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "ncclCommInitRank failed: %s",
                    g_nccl.getErrorString ? g_nccl.getErrorString(nr) : "?");
    }
    return 0;
}

// Peer-memory exchange: every rank exports its receive buffer and flags
// (CUDA IPC), the handles travel over the communicator (an NCCL all-gather
// of 128 bytes per rank), and every rank maps the others'.  Collective:
// all kv_ranks contexts call it.
extern "C" int gemma3_cuda_peer_init(gemma3_cuda_ctx *ctx) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    const int R = ctx->cfg.kv_ranks, me = ctx->cfg.kv_rank;
    if (R < 2 || R > g3::kMaxPeers)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "peer exchange needs 2 <= kv_ranks <= %d", g3::kMaxPeers);
    if (!ctx->comm) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "peer exchange needs gemma3_cuda_comm_init first");
    if (ctx->peer_ready) return 0;
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    const size_t gfloats = 2 * (size_t)R * ctx->cfg.max_batch * kHeads * kPartialStride;
    CU_TRY(cudaMalloc(&ctx->pgather, gfloats * 4));
    CU_TRY(cudaMalloc(&ctx->pflags, 2 * g3::kMaxPeers * sizeof(unsigned)));
    CU_TRY(cudaMalloc(&ctx->pcounter, sizeof(unsigned)));
    CU_TRY(cudaMemsetAsync(ctx->pgather, 0, gfloats * 4, ctx->stream));
    CU_TRY(cudaMemsetAsync(ctx->pflags, 0, 2 * g3::kMaxPeers * sizeof(unsigned), ctx->stream));
    CU_TRY(cudaMemsetAsync(ctx->pcounter, 0, sizeof(unsigned), ctx->stream));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    unsigned char mine[128];
    cudaIpcMemHandle_t hg, hf;
    CU_TRY(cudaIpcGetMemHandle(&hg, ctx->pgather));
    CU_TRY(cudaIpcGetMemHandle(&hf, ctx->pflags));
    memcpy(mine, &hg, 64);
    memcpy(mine + 64, &hf, 64);
    unsigned char *dbuf = nullptr;
    CU_TRY(cudaMalloc(&dbuf, 128 * (R + 1)));
    std::vector<unsigned char> all(128 * (size_t)R);
    int nr = 0;
    cudaError_t ce = cudaMemcpyAsync(dbuf, mine, 128, cudaMemcpyHostToDevice, ctx->stream);
    if (ce == cudaSuccess) nr = g_nccl.allGather(dbuf, dbuf + 128, 128, kNcclInt8, ctx->comm, ctx->stream);
    if (ce == cudaSuccess && nr == 0)
        ce = cudaMemcpyAsync(all.data(), dbuf + 128, 128 * (size_t)R, cudaMemcpyDeviceToHost, ctx->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(ctx->stream);
    cudaFree(dbuf);
    if (nr != 0)
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "ncclAllGather of IPC handles failed: %s",
                    g_nccl.getErrorString ? g_nccl.getErrorString(nr) : "?");
    CU_TRY(ce);
    for (int r = 0; r < R; ++r) {
        if (r == me) {
            ctx->peer_g[r] = ctx->pgather;
            ctx->peer_f[r] = ctx->pflags;
            continue;
        }
        memcpy(&hg, &all[128 * (size_t)r], 64);
        memcpy(&hf, &all[128 * (size_t)r + 64], 64);
        void *pg = nullptr, *pf = nullptr;
        CU_TRY(cudaIpcOpenMemHandle(&pg, hg, cudaIpcMemLazyEnablePeerAccess));
        ctx->peer_g[r] = (float *)pg;
        CU_TRY(cudaIpcOpenMemHandle(&pf, hf, cudaIpcMemLazyEnablePeerAccess));
        ctx->peer_f[r] = (unsigned *)pf;
    }
    ctx->xepoch = 0;
    ctx->peer_ready = ctx->use_peer = true;
    return 0;
}

extern "C" int gemma3_cuda_set_exchange(gemma3_cuda_ctx *ctx, int mode) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    if (mode != GEMMA3_CUDA_XCHG_NCCL && mode != GEMMA3_CUDA_XCHG_PEER)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad exchange mode %d", mode);
    if (mode == GEMMA3_CUDA_XCHG_PEER && !ctx->peer_ready)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "peer exchange not set up (gemma3_cuda_peer_init)");
    if (mode == GEMMA3_CUDA_XCHG_NCCL && !ctx->comm)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "NCCL exchange needs gemma3_cuda_comm_init");
    ctx->use_peer = mode == GEMMA3_CUDA_XCHG_PEER;
    return 0;
}

// ------------------------------------------------------------------ cache utilities
extern "C" int gemma3_cuda_reset(gemma3_cuda_ctx *ctx) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    for (auto &L : ctx->layers)
        CU_TRY(cudaMemsetAsync(L.kv, 0, (size_t)ctx->cfg.max_batch * 2 * kKvHeads * L.rows * kHeadDim * ctx->esz,
                               ctx->stream));
    if (ctx->peer_ready) {
        // peer exchange back to its initial state; every rank resets, with no
        // exchange in flight, so epochs and flags agree again
        CU_TRY(cudaMemsetAsync(ctx->pflags, 0, 2 * g3::kMaxPeers * sizeof(unsigned), ctx->stream));
        CU_TRY(cudaMemsetAsync(ctx->pcounter, 0, sizeof(unsigned), ctx->stream));
        ctx->xepoch = 0;
    }
    return gemma3_cuda_synchronize(ctx);
}

static int cache_args(gemma3_cuda_ctx *ctx, int layer, int seq) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    if (layer < 0 || layer >= ctx->cfg.num_layers) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad layer %d", layer);
    if (seq < 0 || seq >= ctx->cfg.max_batch) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad sequence slot %d", seq);
    return 0;
}

extern "C" int gemma3_cuda_export_cache(gemma3_cuda_ctx *ctx, int layer, int seq, float *k, float *v) {
    if (int r = cache_args(ctx, layer, seq)) return r;
    if (!k || !v) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null buffer");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    const LayerState &L = ctx->layers[layer];
    const size_t plane = (size_t)L.rows * kHeadDim, n = (size_t)L.rows * kKvHeads * kHeadDim;
    float *tmp = nullptr;
    CU_TRY(cudaMalloc(&tmp, n * 4));
    for (int sel = 0; sel < 2; ++sel) {
        const size_t off = ((size_t)seq * 2 + sel) * kKvHeads * plane;
        if (ctx->esz == 2)
            g3::export_rows<__nv_bfloat16><<<592, 256, 0, ctx->stream>>>(
                reinterpret_cast<const __nv_bfloat16 *>(L.kv) + off, plane, L.rows, tmp);
        else
            g3::export_rows<float><<<592, 256, 0, ctx->stream>>>(reinterpret_cast<const float *>(L.kv) + off, plane,
                                                                  L.rows, tmp);
        if (int r = check_launch(ctx, 1)) { cudaFree(tmp); return r; }
        cudaError_t e = cudaMemcpyAsync(sel ? v : k, tmp, n * 4, cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) {
            cudaFree(tmp);
            return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "export: %s", cudaGetErrorString(e));
        }
    }
    cudaFree(tmp);
    return 0;
}

extern "C" int gemma3_cuda_import_cache(gemma3_cuda_ctx *ctx, int layer, int seq, const float *k, const float *v,
                                        int rows) {
    if (int r = cache_args(ctx, layer, seq)) return r;
    const LayerState &L = ctx->layers[layer];
    if (!k || !v || rows < 0 || rows > L.rows) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad import rows %d", rows);
    if (rows == 0) return 0;
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    const size_t plane = (size_t)L.rows * kHeadDim, n = (size_t)rows * kKvHeads * kHeadDim;
    float *tmp = nullptr;
    CU_TRY(cudaMalloc(&tmp, n * 4));
    for (int sel = 0; sel < 2; ++sel) {
        cudaError_t e = cudaMemcpyAsync(tmp, sel ? v : k, n * 4, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) { cudaFree(tmp); return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "import copy"); }
        const size_t off = ((size_t)seq * 2 + sel) * kKvHeads * plane;
        if (ctx->esz == 2)
            g3::import_rows<__nv_bfloat16><<<592, 256, 0, ctx->stream>>>(
                tmp, reinterpret_cast<__nv_bfloat16 *>(L.kv) + off, plane, rows);
        else
            g3::import_rows<float><<<592, 256, 0, ctx->stream>>>(tmp, reinterpret_cast<float *>(L.kv) + off, plane,
                                                                  rows);
        if (int r = check_launch(ctx, 1)) { cudaFree(tmp); return r; }
    }
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "import: %s", cudaGetErrorString(e));
    return 0;
}

extern "C" int gemma3_cuda_fill_cache_random(gemma3_cuda_ctx *ctx, int layer, int seq, int rows, uint64_t seed) {
    if (int r = cache_args(ctx, layer, seq)) return r;
    const LayerState &L = ctx->layers[layer];
    if (rows < 0 || rows > L.rows) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad fill rows %d", rows);
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    const size_t plane = (size_t)L.rows * kHeadDim;
    for (int sel = 0; sel < 2; ++sel)
        for (int h = 0; h < kKvHeads; ++h) {
            const size_t off = (((size_t)seq * 2 + sel) * kKvHeads + h) * plane;
            const uint64_t s = seed * 0x9E3779B97F4A7C15ull + (uint64_t)((layer * 2 + sel) * kKvHeads + h) * 0x632BE59BD9B4E019ull;
            if (ctx->esz == 2)
                g3::fill_normal<__nv_bfloat16><<<296, 256, 0, ctx->stream>>>(
                    reinterpret_cast<__nv_bfloat16 *>(L.kv) + off, (size_t)rows * kHeadDim, s);
            else
                g3::fill_normal<float><<<296, 256, 0, ctx->stream>>>(reinterpret_cast<float *>(L.kv) + off,
                                                                      (size_t)rows * kHeadDim, s);
            if (int r = check_launch(ctx, 1)) return r;
        }
    return 0;
}

// ------------------------------------------------------------------ failure-path self-test
extern "C" int gemma3_cuda_selftest_wait_timeout(gemma3_cuda_ctx *ctx) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    g3::wait_timeout_probe<<<1, 32, 0, ctx->stream>>>(ctx->err);
    if (int r = check_launch(ctx, 1)) return r;
    return gemma3_cuda_synchronize(ctx);  // expected: GEMMA3_CUDA_ERR_GENERATION_FAILED
}

// ------------------------------------------------------------------ profiling
extern "C" int gemma3_cuda_profile(gemma3_cuda_ctx *ctx, int enable) {
    if (!ctx) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null context");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    CU_TRY(cudaStreamSynchronize(ctx->stream));
    ctx->prof = enable != 0;
    ctx->spans.clear();
    ctx->ev_used = 0;
    return 0;
}

extern "C" int gemma3_cuda_profile_read(gemma3_cuda_ctx *ctx, int kernel, long long *launches, double *ms,
                                        double *work) {
    if (!ctx || !launches || !ms || !work) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null argument");
    CU_TRY(cudaSetDevice(ctx->cfg.device));
    CU_TRY(cudaStreamSynchronize(ctx->stream));
    long long n = 0;
    double t = 0, w = 0;
    for (const auto &sp : ctx->spans) {
        if (sp.kind != kernel) continue;
        float f = 0;
        CU_TRY(cudaEventElapsedTime(&f, ctx->ev_pool[sp.e0], ctx->ev_pool[sp.e1]));
        ++n;
        t += f;
        w += sp.work;
    }
    *launches = n;
    *ms = t;
    *work = w;
    return 0;
}

// ------------------------------------------------------------------ decode without allocation
// For callers that cannot allocate device memory: serving loops that may not
// stall on cudaMalloc's implicit device synchronisation, hosts whose memory
// budget is fixed when the process starts, and embedders that hand every
// device buffer in themselves.
// The split-KV decode needs scratch (the scaled queries and the per-split
// (m, l, O) partials); here it lives in one file-scope device array that
// every GPU which loads this library holds until the process exits.
namespace {
constexpr int kNoAllocMaxBatch = 64;
constexpr int kNoAllocMaxSlots = 4096;  // (sequence, head, split) partials
constexpr size_t kNoAllocQ = (size_t)kNoAllocMaxBatch * kHeads * kHeadDim;  // 512 KB
constexpr size_t kNoAllocPart = (size_t)kNoAllocMaxSlots * kPartialStride;  // 4.03 MB
constexpr size_t kNoAllocStatus = 64;                                      // status word + pad
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float *g_noalloc_addr[kNoAllocMaxDevices] = {};
}  // namespace

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocQ + kNoAllocPart + kNoAllocStatus];

// Runs after the merge: a failed device wait in the split kernel (its status
// word is non-zero) turns the whole output into NaN, so a caller that has no
// status channel still cannot read a partial result as a valid one.
__global__ void noalloc_poison_on_error(const unsigned *status, float *out, int n) {
    if (*(volatile const unsigned *)status == 0u) return;
    const float nan = __int_as_float(0x7fc00000);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = nan;
}

__global__ void noalloc_scale_q(const float *__restrict__ q, float *__restrict__ dst, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = q[i] * g3::kScaleLog2;
}

extern "C" int gemma3_cuda_gqa_decode_noalloc(const float *q, const void *kv, int kv_dtype, int rows, int B,
                                              const int *nrows, float *out, void *stream) {
    if (!q || !kv || !nrows || !out) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "null argument");
    // the split kernel streams the cache with 16-byte bulk copies
    if (reinterpret_cast<uintptr_t>(kv) & 15u)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "kv must be 16-byte aligned (bulk copies)");
    if (kv_dtype != GEMMA3_CUDA_KV_F32 && kv_dtype != GEMMA3_CUDA_KV_BF16)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "bad kv_dtype %d", kv_dtype);
    if (B < 1 || B > kNoAllocMaxBatch)
        return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "B=%d outside 1..%d: the no-allocation scratch holds at most %d sequences",
                    B, kNoAllocMaxBatch, kNoAllocMaxBatch);
    if (rows < 1) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "rows must be >= 1");
    int maxrows = 0;
    long long total = 0;
    for (int b = 0; b < B; ++b) {
        if (nrows[b] < 1 || nrows[b] > rows)
            return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "nrows[%d]=%d outside 1..rows=%d", b, nrows[b], rows);
        maxrows = std::max(maxrows, nrows[b]);
        total += (long long)nrows[b] * kKvHeads;
    }
    int dev = 0;
    CU_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(GEMMA3_CUDA_ERR_INVALID_ARG, "device %d unsupported", dev);
    float *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_addr[dev]) {
            // One-time set-up on this device (the current one): resolve the
            // array's device address; the host-side symbol is not it.
            void *p = nullptr;
            CU_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            // same limits the context path sets for the plain form (the
            // attribute is per function)
            const int smem_bf = g3::DecodeCfg<__nv_bfloat16>::NS * 2 * g3::DecodeCfg<__nv_bfloat16>::TK * kHeadDim * 2;
            const int smem_f = g3::DecodeCfg<float>::NS * 2 * g3::DecodeCfg<float>::TK * kHeadDim * 4;
            CU_TRY(cudaFuncSetAttribute(g3::decode_splitkv<__nv_bfloat16, false>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bf));
            CU_TRY(cudaFuncSetAttribute(g3::decode_splitkv<float, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        smem_f));
            g_noalloc_addr[dev] = static_cast<float *>(p);
        }
        scratch = g_noalloc_addr[dev];
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float *qs = scratch;
    float *part = scratch + kNoAllocQ;
    unsigned *status = reinterpret_cast<unsigned *>(scratch + kNoAllocQ + kNoAllocPart);
    // status block: bits, pad, no host mirror (g3::raise_status)
    CU_TRY(cudaMemsetAsync(status, 0, 16, st));

    // Split plan as for the context path, capped by the scratch slots.
    const bool bf = kv_dtype == GEMMA3_CUDA_KV_BF16;
    const int TK = bf ? g3::DecodeCfg<__nv_bfloat16>::TK : g3::DecodeCfg<float>::TK;
    const long long target = 148LL * 8;
    const int max_split = std::max(1, kNoAllocMaxSlots / (B * kHeads));
    long long chunk = std::max<long long>(4 * TK, (total + target - 1) / target);
    chunk = std::max<long long>(chunk, (maxrows + max_split - 1) / max_split);
    chunk = (chunk + TK - 1) / TK * TK;
    const int nsplit = (int)((maxrows + chunk - 1) / chunk);

    const int nq = B * kHeads * kHeadDim;
    noalloc_scale_q<<<(nq + 255) / 256, 256, 0, st>>>(q, qs, nq);

    g3::DecodeRows rws;
    rws.B = B;
    for (int b = 0; b < B; ++b) {
        rws.seq[b] = b;
        rws.nrows[b] = nrows[b];
        rws.pos[b] = 0;
    }
    g3::DecodeParams p;
    p.q = qs;
    p.qraw = p.kraw = p.vraw = nullptr;
    p.eps = 0.f;
    p.tickets = nullptr;
    p.L.kv = const_cast<void *>(kv);
    p.L.rows = rows;
    p.L.is_global = 1;
    p.L.shard_lo = 0;
    p.L.shard_hi = rows;
    p.L.qn = p.L.kn = nullptr;
    p.L.rope = nullptr;
    p.chunk = (int)chunk;
    p.nsplit = nsplit;
    p.partial = part;
    p.out = nullptr;
    p.write_partial = 1;
    p.err = status;
    if (bf) {
        constexpr int smem = g3::DecodeCfg<__nv_bfloat16>::NS * 2 * g3::DecodeCfg<__nv_bfloat16>::TK * kHeadDim * 2;
        g3::decode_splitkv<__nv_bfloat16, false><<<dim3(nsplit, kKvHeads, B), 256, smem, st>>>(p, rws);
    } else {
        constexpr int smem = g3::DecodeCfg<float>::NS * 2 * g3::DecodeCfg<float>::TK * kHeadDim * 4;
        g3::decode_splitkv<float, false><<<dim3(nsplit, kKvHeads, B), 256, smem, st>>>(p, rws);
    }
    const size_t hs = (size_t)nsplit * kPartialStride;
    g3::merge_partials<<<B * kHeads, 256, 0, st>>>(part, nsplit, kHeads * hs, hs, kPartialStride, out, nullptr);
    noalloc_poison_on_error<<<(nq + 1023) / 1024, 256, 0, st>>>(status, out, nq);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(GEMMA3_CUDA_ERR_GENERATION_FAILED, "kernel launch failed: %s", cudaGetErrorString(e));
    return 0;
}
