// GGUF decoder on B200: the llama / qwen2 forward of the reference's GGUF path
// (llama.cpp b4514 behind the bridge of src/gguf-cuda.cu) with every step on the
// device -- embedding lookup, RMSNorm, Q/K/V dequant-GEMV (+ QKV bias for qwen2),
// RoPE (interleaved pairs for llama with llama3 frequency factors, split-half pairs
// for qwen2), the fp32 KV cache, grouped-query attention, O + residual, SwiGLU FFN,
// the tied vocabulary head and the sampler -- captured per token in CUDA graphs.
//
// Semantics follow llama.cpp's graph for these architectures as publicly documented
// (ggml_rms_norm, ggml_rope_ext modes NORM / NEOX with freq factors, soft-max with
// scale 1/sqrt(head_dim)), in fp32 with exactly dequantised weights.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "gguf_kernels.cuh"
#include "mb_common.cuh"
#include "mocha_b200.h"
#include "sampling.cuh"

namespace {

#define TRY(x)                                                                                   \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) {                                                                 \
            fprintf(stderr, "CUDA %s: %d %s\n", #x, (int)e_, cudaGetErrorString(e_));           \
            return 1;                                                                            \
        }                                                                                        \
    } while (0)

// ---- GGUF v3 container ----------------------------------------------------------

struct TensorInfo {
    int type = -1;  // ggml type id (0 = F32)
    int n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;  // from the start of the data section
};

struct Gguf {
    std::unordered_map<std::string, TensorInfo> tensors;
    std::unordered_map<std::string, double> nums;
    std::unordered_map<std::string, std::string> strs;
    size_t data_start = 0;
};

struct Reader {
    const uint8_t *p;
    size_t n, at = 0;
    bool ok = true;
    template <typename T>
    T get()
    {
        T v{};
        if (at + sizeof(T) > n) {
            ok = false;
            return v;
        }
        memcpy(&v, p + at, sizeof(T));
        at += sizeof(T);
        return v;
    }
    std::string str()
    {
        const uint64_t len = get<uint64_t>();
        if (!ok || len > n - at) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char *>(p + at), (size_t)len);
        at += (size_t)len;
        return s;
    }
};

enum { T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 };

bool scalar_size(uint32_t t, size_t *sz)
{
    static const size_t sizes[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (t > T_F64 || t == T_STR || t == T_ARR) return false;
    *sz = sizes[t];
    return true;
}

double read_number(Reader &r, uint32_t t)
{
    switch (t) {
    case T_U8: return r.get<uint8_t>();
    case T_I8: return r.get<int8_t>();
    case T_U16: return r.get<uint16_t>();
    case T_I16: return r.get<int16_t>();
    case T_U32: return r.get<uint32_t>();
    case T_I32: return r.get<int32_t>();
    case T_F32: return r.get<float>();
    case T_BOOL: return r.get<uint8_t>();
    case T_U64: return (double)r.get<uint64_t>();
    case T_I64: return (double)r.get<int64_t>();
    case T_F64: return r.get<double>();
    default: r.ok = false; return 0;
    }
}

bool parse_gguf(const uint8_t *p, size_t n, Gguf *g)
{
    Reader r{p, n};
    if (r.get<uint32_t>() != 0x46554747u) return false;  // "GGUF"
    const uint32_t version = r.get<uint32_t>();
    if (version < 2 || version > 3) return false;
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) return false;
    for (uint64_t i = 0; i < n_kv && r.ok; i++) {
        const std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        if (t == T_STR) {
            g->strs[key] = r.str();
        } else if (t == T_ARR) {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t count = r.get<uint64_t>();
            if (et == T_STR) {
                for (uint64_t j = 0; j < count && r.ok; j++) r.str();
            } else {
                size_t sz;
                if (!scalar_size(et, &sz) || count > (n - r.at) / (sz ? sz : 1)) return false;
                r.at += (size_t)count * sz;
            }
        } else {
            g->nums[key] = read_number(r, t);
        }
    }
    for (uint64_t i = 0; i < n_tensors && r.ok; i++) {
        const std::string name = r.str();
        TensorInfo ti;
        ti.n_dims = (int)r.get<uint32_t>();
        if (ti.n_dims < 1 || ti.n_dims > 4) return false;
        for (int d = 0; d < ti.n_dims; d++) ti.ne[d] = r.get<uint64_t>();
        ti.type = (int)r.get<uint32_t>();
        ti.offset = r.get<uint64_t>();
        g->tensors[name] = ti;
    }
    if (!r.ok) return false;
    const auto al = g->nums.find("general.alignment");
    const size_t align = al == g->nums.end() ? 32 : (size_t)al->second;
    if (!align || (align & (align - 1))) return false;
    g->data_start = (r.at + align - 1) / align * align;
    return g->data_start <= n;
}

size_t tensor_bytes(const TensorInfo &t)
{
    const uint64_t rows = t.ne[1] * t.ne[2] * t.ne[3];
    if (t.type == 0) return (size_t)(t.ne[0] * rows * 4);
    const unsigned rb = gguf::row_bytes(t.type, (int)t.ne[0]);
    return (size_t)rb * rows;
}

// ---- device kernels ---------------------------------------------------------------


struct RopeArgs {
    const float *cos_t, *sin_t;  // [context][head_dim/2]
    int head_dim, heads, kv_heads, neox, context;
};

// The per-token kernels are launched with programmatic stream serialisation: each lets
// the next one launch at once and waits for the previous one before reading anything.
__device__ __forceinline__ void pdl_enter()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename... KArgs, typename... Args>
int pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? 0 : 1;
}

constexpr int kMaxHeadDim = 128;

// QKV post-processing and attention of one query head, split over the positions: CTA
// (h, j) of kFaSplits per head takes positions [j c, j c + c), c = ceil((pos+1)/kFaSplits):
//   post    the head's q and its KV head's k get the biases and RoPE exactly as
//           k_qkv_post computes them, v its bias; the split holding pos keeps k and v in
//           shared memory and, for the first query head of each KV group, writes them to
//           the cache (no split reads a cache row another is writing: the row at pos is
//           used only by its own split);
//   scores  one position per thread: the key row against q (float4 loads), times
//           1/sqrt(head_dim);
//   softmax split max m, exp(s - m) in place, split sum l;
//   P V     warp w takes positions w, w + 8, ...; lane l accumulates dims l + 32 j
//           (coalesced key rows), the 8 warp partials are added in warp order;
//   combine the split writes (m, l, acc) and takes a ticket; the last split of the head
//           adds the splits' acc e^(m - M) / sum l e^(m - M) in split order (M their max)
//           and resets the ticket for the next launch.
// One launch per layer; kFaSplits x heads CTAs instead of one per head (12 for Qwen2.5-1.5B).
constexpr int kFaThreads = 256, kFaWarps = kFaThreads / 32, kFaContext = 1024, kFaSplits = 8;
constexpr int kFaSpan = kFaContext / kFaSplits;  // positions of one split at most

__global__ void __launch_bounds__(kFaThreads)
    k_attention_fused(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                      const float *__restrict__ bq, const float *__restrict__ bk, const float *__restrict__ bv,
                      RopeArgs ra, const int *__restrict__ pos_ptr, float *__restrict__ kc, float *__restrict__ vc,
                      int layer, float *__restrict__ out, float *__restrict__ part, unsigned *__restrict__ ticket)
{
    pdl_enter();
    __shared__ __align__(16) float qs[kMaxHeadDim], kn[kMaxHeadDim];
    __shared__ float vn[kMaxHeadDim];
    __shared__ float sc[kFaSpan];
    __shared__ float red[kFaWarps];
    __shared__ float wacc[kFaWarps][kMaxHeadDim];
    __shared__ int last;
    const int h = blockIdx.x, j = blockIdx.y, hd = ra.head_dim, half = hd / 2, gqa = ra.heads / ra.kv_heads;
    const int kvh = h / gqa;
    const int pos = min(*pos_ptr, ra.context - 1), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int chunk = (pos + kFaSplits) / kFaSplits, p0 = j * chunk, p1 = min(pos + 1, p0 + chunk);
    const bool holds_pos = p0 <= pos && pos < p1;
    const bool writer = h % gqa == 0 && holds_pos;
    const size_t row = ((size_t)layer * ra.kv_heads + kvh) * ra.context;
    if (tid < half) {
        // NORM: pairs (2i, 2i+1); NEOX: pairs (i, i + half)
        const int i = tid, a = ra.neox ? i : 2 * i, b = ra.neox ? a + half : a + 1;
        const float cs = ra.cos_t[pos * half + i], sn = ra.sin_t[pos * half + i];
        float x0 = q[h * hd + a], x1 = q[h * hd + b];
        if (bq) {
            x0 += bq[h * hd + a];
            x1 += bq[h * hd + b];
        }
        qs[a] = x0 * cs - x1 * sn;
        qs[b] = x0 * sn + x1 * cs;
        if (holds_pos) {
            x0 = k[kvh * hd + a];
            x1 = k[kvh * hd + b];
            if (bk) {
                x0 += bk[kvh * hd + a];
                x1 += bk[kvh * hd + b];
            }
            const float y0 = x0 * cs - x1 * sn, y1 = x0 * sn + x1 * cs;
            kn[a] = y0;
            kn[b] = y1;
            if (writer) {
                float *kd = kc + (row + pos) * hd;
                kd[a] = y0;
                kd[b] = y1;
            }
        }
    }
    if (tid < hd && holds_pos) {
        const float vv = v[kvh * hd + tid] + (bv ? bv[kvh * hd + tid] : 0.f);
        vn[tid] = vv;
        if (writer) vc[(row + pos) * hd + tid] = vv;
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf((float)hd);
    const float *kb = kc + row * hd, *vb = vc + row * hd;
    float mloc = -INFINITY;
    for (int p = p0 + tid; p < p1; p += kFaThreads) {
        const float4 *kr = reinterpret_cast<const float4 *>(p == pos ? kn : kb + (size_t)p * hd);
        const float4 *qr = reinterpret_cast<const float4 *>(qs);
        float z = 0.f;
        for (int jj = 0; jj < hd / 4; jj++) {
            const float4 kv = kr[jj], qv = qr[jj];
            z = fmaf(qv.x, kv.x, z);
            z = fmaf(qv.y, kv.y, z);
            z = fmaf(qv.z, kv.z, z);
            z = fmaf(qv.w, kv.w, z);
        }
        z *= scale;
        sc[p - p0] = z;
        mloc = fmaxf(mloc, z);
    }
    mloc = mb::warp_max(mloc);
    if (lane == 0) red[warp] = mloc;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int w = 1; w < kFaWarps; w++) m = fmaxf(m, red[w]);
    __syncthreads();  // red is reused for the sums
    float lloc = 0.f;
    for (int p = p0 + tid; p < p1; p += kFaThreads) {
        const float e = expf(sc[p - p0] - m);
        sc[p - p0] = e;
        lloc += e;
    }
    lloc = mb::warp_sum(lloc);
    if (lane == 0) red[warp] = lloc;
    __syncthreads();
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kFaWarps; w++) l += red[w];
    const int per = hd / 32;  // dims per lane (2 or 4)
    float acc[kMaxHeadDim / 32];
#pragma unroll
    for (int jj = 0; jj < kMaxHeadDim / 32; jj++) acc[jj] = 0.f;
    for (int p = p0 + warp; p < p1; p += kFaWarps) {
        const float e = sc[p - p0];
        const float *vr = p == pos ? vn : vb + (size_t)p * hd;
#pragma unroll
        for (int jj = 0; jj < kMaxHeadDim / 32; jj++)
            if (jj < per) acc[jj] = fmaf(e, vr[lane + 32 * jj], acc[jj]);
    }
#pragma unroll
    for (int jj = 0; jj < kMaxHeadDim / 32; jj++)
        if (jj < per) wacc[warp][lane + 32 * jj] = acc[jj];
    __syncthreads();
    // this split's (m, l, unnormalised output), then the ticket
    float *mine = part + ((size_t)h * kFaSplits + j) * (kMaxHeadDim + 2);
    for (int d = tid; d < hd; d += kFaThreads) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < kFaWarps; w++) a += wacc[w][d];
        mine[2 + d] = a;
    }
    if (tid == 0) {
        mine[0] = m;  // -inf for an empty split (l = 0)
        mine[1] = l;
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        last = atomicAdd(ticket + h, 1u) == (unsigned)(kFaSplits - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float *hp = part + (size_t)h * kFaSplits * (kMaxHeadDim + 2);
    float M = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < kFaSplits; jj++) M = fmaxf(M, __ldcg(hp + jj * (kMaxHeadDim + 2)));
    float L = 0.f, f[kFaSplits];
#pragma unroll
    for (int jj = 0; jj < kFaSplits; jj++) {
        const float ms = __ldcg(hp + jj * (kMaxHeadDim + 2));
        f[jj] = ms == -INFINITY ? 0.f : expf(ms - M);
        L = fmaf(f[jj], __ldcg(hp + jj * (kMaxHeadDim + 2) + 1), L);
    }
    for (int d = tid; d < hd; d += kFaThreads) {
        float a = 0.f;
#pragma unroll
        for (int jj = 0; jj < kFaSplits; jj++)
            if (f[jj] != 0.f) a = fmaf(f[jj], __ldcg(hp + jj * (kMaxHeadDim + 2) + 2 + d), a);
        out[h * hd + d] = a / L;
    }
    if (tid == 0) ticket[h] = 0u;  // every split of this launch has taken its ticket
}

__global__ void k_swiglu(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ h, int n)
{
    pdl_enter();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float x = g[i];
        h[i] = (x / (1.0f + expf(-x))) * u[i];
    }
}

__global__ void k_gguf_advance(int *state /* token, pos */, const int *prompt)
{
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        state[1]++;
        state[0] = prompt[state[1]];
    }
}

int launch_ok(const char *what)
{
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA %s: %d %s\n", what, (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

struct Layer {
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
    gguf::DevMat q{}, k{}, v{}, o{}, gate{}, up{}, down{};
    gguf::MmaMat mq{}, mk{}, mv{}, mo{}, mgate{}, mup{}, mdown{};  // tensor-core layout
};

}  // namespace

struct mocha_gguf {
    int device = 0;
    cudaStream_t stream = nullptr;
    mocha_gguf_info info{};
    std::vector<uint8_t *> allocs;
    std::vector<Layer> layers;
    gguf::DevMat embd{};
    gguf::MmaMat membd{};  // the tied head in the tensor-core layout
    bool mma = true;       // GEMVs on the tensor cores (MOCHA_B200_GGUF_GEMV=cuda: CUDA cores)
    const float *out_norm = nullptr;
    RopeArgs rope{};
    float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *g = nullptr,
          *u = nullptr, *h = nullptr, *logits = nullptr, *kc = nullptr, *vc = nullptr;
    float *apart = nullptr;      // attention split partials [heads][kFaSplits][head_dim max + 2]
    unsigned *aticket = nullptr; // attention splits done per head (reset by the last split)
    int *state = nullptr;     // device [token, pos]
    int *h_state = nullptr;   // pinned staging
    int *prompt = nullptr;
    sampling::SeqState *seq = nullptr;
    sampling::Params *params = nullptr, *h_params = nullptr;
    unsigned long long *scratch = nullptr, *keys = nullptr;
    int *h_out = nullptr, *h_out_count = nullptr, *d_out = nullptr, *d_out_count = nullptr;
    cudaGraphExec_t g_forward[2] = {nullptr, nullptr}, g_prefill = nullptr, g_decode = nullptr;
    cudaEvent_t ev[4] = {};
    unsigned long long launches_per_token = 0;
};

namespace {

int dev_alloc(mocha_gguf *m, void **p, size_t bytes)
{
    TRY(cudaMalloc(p, bytes));
    m->allocs.push_back((uint8_t *)*p);
    return 0;
}

// One forward step for the token/pos in m->state; project: final norm + head.
int enqueue_forward(mocha_gguf *m, bool project)
{
    const mocha_gguf_info &in = m->info;
    const cudaStream_t s = m->stream;
    int rc = gguf::enqueue_dequant_row(m->embd, m->state, m->x, s);
    auto multi = [&](std::initializer_list<std::pair<const gguf::DevMat *, float *>> mats, const float *x,
                     const float *gain, bool accumulate) {
        gguf::MultiGemv g{};
        int i = 0, rows = 0;
        for (auto &mt : mats) {
            g.m[i] = *mt.first;
            g.y[i] = mt.second;
            rows += mt.first->rows;
            g.row_end[i] = rows;
            i++;
        }
        g.n = i;
        g.cols = mats.begin()->first->cols;
        g.accumulate = accumulate ? 1 : 0;
        g.x = x;
        g.gain = gain;
        g.eps = in.eps;
        return gguf::enqueue_gemv_multi(g, s);
    };
    auto mmv = [&](std::initializer_list<std::pair<const gguf::MmaMat *, float *>> mats, const float *x,
                   const float *gain, bool accumulate, const float *up = nullptr) {
        gguf::MultiGemvMma g{};
        int i = 0;
        for (auto &mt : mats) {
            g.m[i] = *mt.first;
            g.y[i] = mt.second;
            i++;
        }
        g.n = i;
        g.cols = mats.begin()->first->cols;
        g.accumulate = accumulate ? 1 : 0;
        g.x = x;
        g.gain = gain;
        g.up = up;
        g.eps = in.eps;
        return gguf::enqueue_gemv_mma(g, s);
    };
    const bool tc = m->mma;
    for (int l = 0; l < in.layers && !rc; l++) {
        const Layer &L = m->layers[l];
        // RMSNorm folded into the fused q|k|v GEMV
        rc = (tc ? mmv({{&L.mq, m->q}, {&L.mk, m->k}, {&L.mv, m->v}}, m->x, L.attn_norm, false)
                 : multi({{&L.q, m->q}, {&L.k, m->k}, {&L.v, m->v}}, m->x, L.attn_norm, false)) ||
             pdl(k_attention_fused, dim3(in.heads, kFaSplits), dim3(kFaThreads), s, m->q, m->k, m->v, L.bq, L.bk,
                 L.bv, m->rope, m->state + 1, m->kc, m->vc, l, m->att, m->apart, m->aticket) ||
             (tc ? mmv({{&L.mo, m->x}}, m->att, nullptr, true) : multi({{&L.o, m->x}}, m->att, nullptr, true)) ||
             (tc ? mmv({{&L.mgate, m->g}, {&L.mup, m->u}}, m->x, L.ffn_norm, false)
                 : multi({{&L.gate, m->g}, {&L.up, m->u}}, m->x, L.ffn_norm, false)) ||
             (tc ? mmv({{&L.mdown, m->x}}, m->g, nullptr, true, m->u)
                 : pdl(k_swiglu, dim3((in.ffn + 255) / 256), dim3(256), s, m->g, m->u, m->h, in.ffn) ||
                       multi({{&L.down, m->x}}, m->h, nullptr, true));
    }
    if (!rc && project)
        rc = tc ? mmv({{&m->membd, m->logits}}, m->x, m->out_norm, false)
                : multi({{&m->embd, m->logits}}, m->x, m->out_norm, false);
    return rc || launch_ok("gguf forward");
}

int capture(mocha_gguf *m, cudaGraphExec_t *out, int kind)
{
    cudaGraph_t g = nullptr;
    TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_forward(m, kind == 1 || kind == 3);
    if (!rc && kind == 2) k_gguf_advance<<<1, 1, 0, m->stream>>>(m->state, m->prompt);
    if (!rc && kind == 3) {
        rc = sampling::enqueue_topk(m->logits, m->info.vocab, m->seq->history, &m->seq->history_count, m->params,
                                    m->scratch, m->keys, m->stream) ||
             sampling::enqueue_sample(m->keys, m->params, m->seq, m->state, m->state + 1, m->d_out, m->d_out_count,
                                      m->stream);
    }
    const cudaError_t end = cudaStreamEndCapture(m->stream, &g);
    if (rc || end != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        fprintf(stderr, "CUDA gguf graph capture failed\n");
        return 1;
    }
    const cudaError_t inst = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    TRY(inst);
    return 0;
}

void release(mocha_gguf *m)
{
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    cudaGraphExec_t gs[] = {m->g_forward[0], m->g_forward[1], m->g_prefill, m->g_decode};
    for (auto g : gs)
        if (g) cudaGraphExecDestroy(g);
    for (auto e : m->ev)
        if (e) cudaEventDestroy(e);
    for (auto p : m->allocs) cudaFree(p);
    void *host[] = {m->h_state, m->h_params, m->h_out, m->h_out_count};
    for (void *p : host)
        if (p) cudaFreeHost(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int upload_matrix(mocha_gguf *m, const Gguf &g, const uint8_t *file, const std::string &name, int rows, int cols,
                  gguf::DevMat *out, uint8_t *staging, gguf::MmaMat *mma = nullptr)
{
    const auto it = g.tensors.find(name);
    if (it == g.tensors.end()) {
        fprintf(stderr, "MOCHA_B200: GGUF tensor %s missing\n", name.c_str());
        return 1;
    }
    const TensorInfo &t = it->second;
    if ((int)t.ne[0] != cols || (int)t.ne[1] != rows || !gguf::row_bytes(t.type, cols) ||
        (t.type != gguf::Q4_K && t.type != gguf::Q6_K && t.type != gguf::Q8_0) || cols % 256) {
        fprintf(stderr, "MOCHA_B200: GGUF tensor %s has unsupported type/shape\n", name.c_str());
        return 1;
    }
    const size_t bytes = tensor_bytes(t);
    uint8_t *dst = nullptr;
    if (dev_alloc(m, (void **)&dst, bytes)) return 1;
    TRY(cudaMemcpyAsync(staging, file + g.data_start + t.offset, bytes, cudaMemcpyHostToDevice, m->stream));
    if (gguf::enqueue_repack(t.type, staging, rows, cols, dst, m->stream)) return 1;
    if (mma) {
        const size_t mb = gguf::mma_bytes(t.type, rows, cols);
        uint8_t *mdst = nullptr;
        if (!mb || dev_alloc(m, (void **)&mdst, mb)) return 1;
        if (gguf::enqueue_repack_mma(t.type, staging, rows, cols, mdst, m->stream)) return 1;
        *mma = gguf::MmaMat{t.type, rows, cols, mdst};
    }
    TRY(cudaStreamSynchronize(m->stream));
    *out = gguf::make_devmat(t.type, rows, cols, dst);
    return 0;
}

int upload_f32(mocha_gguf *m, const Gguf &g, const uint8_t *file, const std::string &name, int n, const float **out,
               bool optional)
{
    const auto it = g.tensors.find(name);
    if (it == g.tensors.end()) {
        if (optional) {
            *out = nullptr;
            return 0;
        }
        fprintf(stderr, "MOCHA_B200: GGUF tensor %s missing\n", name.c_str());
        return 1;
    }
    if (it->second.type != 0 || (int)it->second.ne[0] != n) {
        fprintf(stderr, "MOCHA_B200: GGUF tensor %s is not f32[%d]\n", name.c_str(), n);
        return 1;
    }
    float *dst = nullptr;
    if (dev_alloc(m, (void **)&dst, sizeof(float) * n)) return 1;
    TRY(cudaMemcpy(dst, file + g.data_start + it->second.offset, sizeof(float) * n, cudaMemcpyHostToDevice));
    *out = dst;
    return 0;
}

int open_model(mocha_gguf *m, int device, const uint8_t *file, size_t bytes)
{
    cudaDeviceProp prop;
    TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) {
        fprintf(stderr, "MOCHA_B200: requires a compute capability 10.x (B200) device\n");
        return 1;
    }
    m->device = device;
    TRY(cudaSetDevice(device));
    TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    for (auto &e : m->ev) TRY(cudaEventCreate(&e));
    Gguf g;
    if (!parse_gguf(file, bytes, &g)) {
        fprintf(stderr, "MOCHA_B200: not a GGUF v2/v3 file\n");
        return 1;
    }
    for (const auto &t : g.tensors)
        if (g.data_start + t.second.offset + tensor_bytes(t.second) > bytes) {
            fprintf(stderr, "MOCHA_B200: GGUF tensor %s out of range\n", t.first.c_str());
            return 1;
        }
    const std::string arch = g.strs.count("general.architecture") ? g.strs["general.architecture"] : "";
    mocha_gguf_info &in = m->info;
    if (arch == "llama") in.arch = 0;
    else if (arch == "qwen2") in.arch = 1;
    else {
        fprintf(stderr, "MOCHA_B200: GGUF architecture '%s' not supported (llama, qwen2)\n", arch.c_str());
        return 1;
    }
    auto num = [&](const char *key, double dflt) {
        const auto it = g.nums.find(arch + "." + key);
        return it == g.nums.end() ? dflt : it->second;
    };
    in.layers = (int)num("block_count", 0);
    in.dim = (int)num("embedding_length", 0);
    in.ffn = (int)num("feed_forward_length", 0);
    in.heads = (int)num("attention.head_count", 0);
    in.kv_heads = (int)num("attention.head_count_kv", in.heads);
    in.eps = (float)num("attention.layer_norm_rms_epsilon", 1e-5);
    in.rope_base = (float)num("rope.freq_base", 10000.0);
    in.context = (int)num("context_length", 1024);
    // the reference engines run a 1024 context; k_attention_fused keeps one score per
    // position of it in shared memory
    static_assert(kFaContext >= 1024, "attention score buffer shorter than the context");
    if (in.context > 1024 || in.context < 1) in.context = 1024;
    const auto te = g.tensors.find("token_embd.weight");
    if (te == g.tensors.end() || in.layers < 1 || in.dim < 256 || in.heads < 1 || in.kv_heads < 1 ||
        in.heads % in.kv_heads || in.dim % in.heads) {
        fprintf(stderr, "MOCHA_B200: incomplete GGUF hyper-parameters\n");
        return 1;
    }
    in.vocab = (int)te->second.ne[1];
    in.head_dim = in.dim / in.heads;
    in.rope_neox = in.arch == 1;
    if (in.head_dim % 32 || in.head_dim > kMaxHeadDim || in.ffn % 256 || in.dim % 256) {
        fprintf(stderr, "MOCHA_B200: unsupported GGUF shapes\n");
        return 1;
    }
    in.eos = g.nums.count("tokenizer.ggml.eos_token_id") ? (int)g.nums["tokenizer.ggml.eos_token_id"] : -1;
    const int dim = in.dim, kvd = in.kv_heads * in.head_dim;
    // staging for raw tensors before the device-layout repack
    size_t max_raw = 0;
    for (const auto &t : g.tensors) max_raw = max_raw > tensor_bytes(t.second) ? max_raw : tensor_bytes(t.second);
    uint8_t *staging = nullptr;
    TRY(cudaMalloc(&staging, max_raw));
    const char *gemv = getenv("MOCHA_B200_GGUF_GEMV");
    m->mma = !(gemv && !strcmp(gemv, "cuda"));
    int rc = upload_matrix(m, g, file, "token_embd.weight", in.vocab, dim, &m->embd, staging,
                           m->mma ? &m->membd : nullptr);
    rc = rc || upload_f32(m, g, file, "output_norm.weight", dim, &m->out_norm, false);
    m->layers.resize(in.layers);
    for (int l = 0; l < in.layers && !rc; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        Layer &L = m->layers[l];
        rc = upload_f32(m, g, file, p + "attn_norm.weight", dim, &L.attn_norm, false) ||
             upload_f32(m, g, file, p + "ffn_norm.weight", dim, &L.ffn_norm, false) ||
             upload_f32(m, g, file, p + "attn_q.bias", dim, &L.bq, true) ||
             upload_f32(m, g, file, p + "attn_k.bias", kvd, &L.bk, true) ||
             upload_f32(m, g, file, p + "attn_v.bias", kvd, &L.bv, true) ||
             upload_matrix(m, g, file, p + "attn_q.weight", dim, dim, &L.q, staging, m->mma ? &L.mq : nullptr) ||
             upload_matrix(m, g, file, p + "attn_k.weight", kvd, dim, &L.k, staging, m->mma ? &L.mk : nullptr) ||
             upload_matrix(m, g, file, p + "attn_v.weight", kvd, dim, &L.v, staging, m->mma ? &L.mv : nullptr) ||
             upload_matrix(m, g, file, p + "attn_output.weight", dim, dim, &L.o, staging, m->mma ? &L.mo : nullptr) ||
             upload_matrix(m, g, file, p + "ffn_gate.weight", in.ffn, dim, &L.gate, staging,
                           m->mma ? &L.mgate : nullptr) ||
             upload_matrix(m, g, file, p + "ffn_up.weight", in.ffn, dim, &L.up, staging, m->mma ? &L.mup : nullptr) ||
             upload_matrix(m, g, file, p + "ffn_down.weight", dim, in.ffn, &L.down, staging,
                           m->mma ? &L.mdown : nullptr);
    }
    cudaFree(staging);
    if (rc) return 1;
    // RoPE tables: theta = pos * base^(-2i/head_dim) / freq_factor[i] (rope_freqs.weight)
    std::vector<float> ff(in.head_dim / 2, 1.0f);
    const auto rf = g.tensors.find("rope_freqs.weight");
    if (rf != g.tensors.end()) {
        if (rf->second.type != 0 || (int)rf->second.ne[0] != in.head_dim / 2) {
            fprintf(stderr, "MOCHA_B200: rope_freqs.weight has the wrong shape\n");
            return 1;
        }
        memcpy(ff.data(), file + g.data_start + rf->second.offset, sizeof(float) * ff.size());
        in.rope_factors = 1;
    }
    const int half = in.head_dim / 2;
    std::vector<float> tab((size_t)in.context * half * 2);
    for (int pos = 0; pos < in.context; pos++)
        for (int i = 0; i < half; i++) {
            const float theta = pos * powf(in.rope_base, -2.0f * i / in.head_dim) / ff[i];
            tab[(size_t)pos * half + i] = cosf(theta);
            tab[(size_t)in.context * half + (size_t)pos * half + i] = sinf(theta);
        }
    float *dtab = nullptr;
    if (dev_alloc(m, (void **)&dtab, sizeof(float) * tab.size())) return 1;
    TRY(cudaMemcpy(dtab, tab.data(), sizeof(float) * tab.size(), cudaMemcpyHostToDevice));
    m->rope = RopeArgs{dtab, dtab + (size_t)in.context * half, in.head_dim, in.heads, in.kv_heads, in.rope_neox,
                       in.context};
    // activations, KV cache, sampler state
    const size_t kv_elems = (size_t)in.layers * in.kv_heads * in.context * in.head_dim;
    if (dev_alloc(m, (void **)&m->x, sizeof(float) * dim) || dev_alloc(m, (void **)&m->xn, sizeof(float) * dim) ||
        dev_alloc(m, (void **)&m->q, sizeof(float) * dim) || dev_alloc(m, (void **)&m->k, sizeof(float) * kvd) ||
        dev_alloc(m, (void **)&m->v, sizeof(float) * kvd) || dev_alloc(m, (void **)&m->att, sizeof(float) * dim) ||
        dev_alloc(m, (void **)&m->g, sizeof(float) * in.ffn) || dev_alloc(m, (void **)&m->u, sizeof(float) * in.ffn) ||
        dev_alloc(m, (void **)&m->h, sizeof(float) * in.ffn) ||
        dev_alloc(m, (void **)&m->logits, sizeof(float) * in.vocab) ||
        dev_alloc(m, (void **)&m->kc, sizeof(float) * kv_elems) ||
        dev_alloc(m, (void **)&m->vc, sizeof(float) * kv_elems) || dev_alloc(m, (void **)&m->state, sizeof(int) * 2) ||
        dev_alloc(m, (void **)&m->apart, sizeof(float) * in.heads * kFaSplits * (kMaxHeadDim + 2)) ||
        dev_alloc(m, (void **)&m->aticket, sizeof(unsigned) * in.heads) ||
        dev_alloc(m, (void **)&m->prompt, sizeof(int) * in.context) ||
        dev_alloc(m, (void **)&m->seq, sizeof(sampling::SeqState)) ||
        dev_alloc(m, (void **)&m->params, sizeof(sampling::Params)) ||
        dev_alloc(m, (void **)&m->scratch, sizeof(unsigned long long) * sampling::kStage1Blocks * sampling::kMaxK) ||
        dev_alloc(m, (void **)&m->keys, sizeof(unsigned long long) * sampling::kMaxK))
        return 1;
    TRY(cudaMemset(m->kc, 0, sizeof(float) * kv_elems));
    TRY(cudaMemset(m->vc, 0, sizeof(float) * kv_elems));
    TRY(cudaMemset(m->aticket, 0, sizeof(unsigned) * in.heads));  // the attention splits' tickets
    TRY(cudaMallocHost(&m->h_state, sizeof(int) * 2));
    TRY(cudaMallocHost(&m->h_params, sizeof(sampling::Params)));
    TRY(cudaHostAlloc(&m->h_out, sizeof(int) * sampling::kOutRing, cudaHostAllocMapped));
    TRY(cudaHostAlloc(&m->h_out_count, sizeof(int), cudaHostAllocMapped));
    TRY(cudaHostGetDevicePointer(&m->d_out, m->h_out, 0));
    TRY(cudaHostGetDevicePointer(&m->d_out_count, m->h_out_count, 0));
    if (sampling::init_device()) return 1;
    if (capture(m, &m->g_forward[0], 0) || capture(m, &m->g_forward[1], 1) || capture(m, &m->g_prefill, 2) ||
        capture(m, &m->g_decode, 3))
        return 1;
    // embedding row, per layer q|k|v, post, attention, O, gate|up, (SwiGLU,) down; head; sampler
    m->launches_per_token = 1 + (unsigned long long)in.layers * (m->mma ? 5 : 6) + 1 + 3;
    TRY(cudaStreamSynchronize(m->stream));
    return 0;
}

}  // namespace

extern "C" int mocha_gguf_open(int device, const void *file, unsigned long long bytes, mocha_gguf **out)
{
    if (!file || !out || bytes < 32) return 1;
    mocha_gguf *m = new mocha_gguf();
    if (open_model(m, device, (const uint8_t *)file, (size_t)bytes)) {
        release(m);
        return 1;
    }
    *out = m;
    return 0;
}

extern "C" int mocha_gguf_close(mocha_gguf *m)
{
    if (!m) return 1;
    release(m);
    return 0;
}

extern "C" int mocha_gguf_get_info(mocha_gguf *m, mocha_gguf_info *info)
{
    if (!m || !info) return 1;
    *info = m->info;
    return 0;
}

extern "C" int mocha_gguf_forward(mocha_gguf *m, int token, int pos, int project, float *logits)
{
    if (!m || token < 0 || token >= m->info.vocab || pos < 0 || pos >= m->info.context) return 1;
    TRY(cudaSetDevice(m->device));
    m->h_state[0] = token;
    m->h_state[1] = pos;
    TRY(cudaMemcpyAsync(m->state, m->h_state, sizeof(int) * 2, cudaMemcpyHostToDevice, m->stream));
    TRY(cudaGraphLaunch(m->g_forward[project ? 1 : 0], m->stream));
    if (project && logits)
        TRY(cudaMemcpyAsync(logits, m->logits, sizeof(float) * m->info.vocab, cudaMemcpyDeviceToHost, m->stream));
    TRY(cudaStreamSynchronize(m->stream));
    return gguf::gemv_take_timeout();
}

namespace {

int begin(mocha_gguf *m, const int *prompt, int n_prompt, const mocha_sampling *s)
{
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= m->info.vocab) return 1;
    TRY(cudaSetDevice(m->device));
    TRY(cudaStreamSynchronize(m->stream));
    sampling::SeqState seq;
    memset(&seq, 0, sizeof seq);
    const int first = n_prompt > sampling::kHistory ? n_prompt - sampling::kHistory : 0;
    for (int i = first; i < n_prompt; i++) seq.history[i - first] = prompt[i];
    seq.history_count = n_prompt - first;
    seq.history_head = seq.history_count % sampling::kHistory;
    seq.seed = s->seed;
    sampling::Params *p = m->h_params;
    p->penalty = s->repeat_penalty;
    p->temperature = s->temperature;
    p->top_k = s->temperature == 0.f ? 1 : s->top_k;
    p->top_p = s->top_p;
    p->eos = m->info.eos;
    p->control_first = m->info.vocab;  // no control-token mask on the GGUF path
    p->vocab = m->info.vocab;
    m->h_state[0] = prompt[0];
    m->h_state[1] = 0;
    TRY(cudaMemcpyAsync(m->seq, &seq, sizeof seq, cudaMemcpyHostToDevice, m->stream));
    TRY(cudaMemcpyAsync(m->params, p, sizeof *p, cudaMemcpyHostToDevice, m->stream));
    TRY(cudaMemcpyAsync(m->prompt, prompt, sizeof(int) * n_prompt, cudaMemcpyHostToDevice, m->stream));
    TRY(cudaMemcpyAsync(m->state, m->h_state, sizeof(int) * 2, cudaMemcpyHostToDevice, m->stream));
    TRY(cudaStreamSynchronize(m->stream));
    *m->h_out_count = 0;
    return 0;
}

}  // namespace

extern "C" int mocha_gguf_generate(mocha_gguf *m, const int *prompt, int n_prompt, int n_new, const mocha_sampling *s,
                                   int *out_tokens, int *n_out, mocha_timing *timing)
{
    if (!m || !prompt || !s || !out_tokens || n_prompt < 1 || n_new < 1 || n_prompt + n_new > m->info.context ||
        !(s->temperature >= 0.f) || !(s->repeat_penalty >= 1.f) ||
        (s->temperature > 0.f && (s->top_k < 1 || s->top_k > sampling::kMaxK)) || !(s->top_p > 0.f && s->top_p <= 1.f))
        return 1;
    if (begin(m, prompt, n_prompt, s)) return 1;
    TRY(cudaEventRecord(m->ev[0], m->stream));
    for (int p = 0; p + 1 < n_prompt; p++) TRY(cudaGraphLaunch(m->g_prefill, m->stream));
    TRY(cudaEventRecord(m->ev[1], m->stream));
    TRY(cudaGraphLaunch(m->g_decode, m->stream));
    TRY(cudaEventRecord(m->ev[2], m->stream));
    for (int i = 1; i < n_new; i++) TRY(cudaGraphLaunch(m->g_decode, m->stream));
    TRY(cudaEventRecord(m->ev[3], m->stream));
    TRY(cudaStreamSynchronize(m->stream));
    if (gguf::gemv_take_timeout()) return 1;
    int n = 0;
    for (int i = 0; i < n_new; i++) out_tokens[i] = m->h_out[i];
    while (n < n_new && out_tokens[n] != m->info.eos) n++;
    if (n_out) *n_out = n;
    if (timing) {
        float a = 0, b = 0;
        TRY(cudaEventElapsedTime(&a, m->ev[0], m->ev[1]));
        TRY(cudaEventElapsedTime(&b, m->ev[2], m->ev[3]));
        timing->prefill_s = a * 1e-3;
        timing->decode_s = b * 1e-3;
        timing->generated = n;
    }
    return 0;
}

extern "C" int mocha_gguf_bench_decode(mocha_gguf *m, int token, int pos0, int pos_end, int warmup, int steps,
                                       float *ms)
{
    if (!m || !ms || token < 0 || token >= m->info.vocab || pos0 < 0 || pos_end <= pos0 || pos_end > m->info.context ||
        warmup < 0 || steps < 1)
        return 1;
    TRY(cudaSetDevice(m->device));
    mocha_sampling greedy{0.f, 1, 1.f, 1.f, 1u};
    int dummy = token;
    if (begin(m, &dummy, 1, &greedy)) return 1;
    m->h_state[0] = token;
    m->h_state[1] = pos0;
    TRY(cudaMemcpyAsync(m->state, m->h_state, sizeof(int) * 2, cudaMemcpyHostToDevice, m->stream));
    int pos = pos0;
    for (int i = 0; i < warmup + steps; i++) {
        if (i == warmup) TRY(cudaEventRecord(m->ev[0], m->stream));
        if (pos == pos_end) {
            TRY(cudaMemcpyAsync(m->state + 1, m->h_state + 1, sizeof(int), cudaMemcpyHostToDevice, m->stream));
            pos = pos0;
        }
        TRY(cudaGraphLaunch(m->g_decode, m->stream));
        pos++;
    }
    TRY(cudaEventRecord(m->ev[1], m->stream));
    TRY(cudaStreamSynchronize(m->stream));
    TRY(cudaEventElapsedTime(ms, m->ev[0], m->ev[1]));
    return gguf::gemv_take_timeout();
}

extern "C" int mocha_gguf_launches_per_step(mocha_gguf *m) { return m ? (int)m->launches_per_token : 0; }
