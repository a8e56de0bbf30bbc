// glm.c's runtime checkpoint (.bin) straight to the device: the file is
// mapped read-only, its header checked and every tensor's offset computed
// as glm.c's runtime_open does (infer.c:357-744), and the tensors uploaded
// through the library's own upload calls. Replaces runtime_open +
// glm_backend_init (backend.c:73-86) for the cuda backend.
//
// Layout (format of glm47_flash_export.py:681-819, read by infer.c):
//   256-byte header (RuntimeConfig, model.h:7-45)
//   output norm, tok_q, tok_s, out_q, out_s          (offsets in the header)
//   layer-0 dense FFN                                (offsets in the header)
//   layer-0 MLA attention (v4 extension; also repeated below)
//   attention of every layer 0..L-1, 15 tensors each (LayerAttnWeights order)
//   shared expert + router of MoE layers 1..L-1     (LayerMoeShared order)
//   routed experts of MoE layers 1..L-1             (LayerMoeRouted order)
#include <cstdint>
#include <cstdio>
#include <cstring>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "glm_cuda.h"
#include "glm_internal.h"

namespace {

// The header as the file stores it (little-endian, the field order and
// widths of RuntimeConfig, model.h:7-45; a binary format, so kept alike).
#pragma pack(push, 4)
struct BinHeader {
    uint32_t magic, version;
    int32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, rope_dim, q_lora_rank,
        kv_lora_rank, kv_mqa_width, n_routed_experts, n_experts_used, n_shared_experts, bos_id, eos_id;
    uint64_t group_size, off_norm, off_tok_q, off_tok_s, off_out_q, off_out_s, total_bytes, off_l0_ffn_norm,
        off_l0_ffn_gate_q, off_l0_ffn_gate_s, off_l0_ffn_up_q, off_l0_ffn_up_s, off_l0_ffn_down_q, off_l0_ffn_down_s;
    int32_t l0_qk_nope_dim, l0_head_k_dim, l0_v_head_dim, l0_flags, moe_ffn_dim;
};
#pragma pack(pop)
static_assert(sizeof(BinHeader) == 204, "checkpoint header layout");

constexpr uint32_t kMagic = 0x67343763u;  // "g47c"
constexpr size_t kHeaderBytes = 256;
constexpr int32_t kFlagAllAttn = 1;

struct Mapped {
    const unsigned char* data = nullptr;
    size_t size = 0;
    ~Mapped() {
        if (data) munmap(const_cast<unsigned char*>(data), size);
    }
};

// Sequential reader over the mapped file: each take() hands out the next
// tensor and fails if it would run past the end.
struct Cursor {
    const unsigned char* base;
    size_t size, off;
    bool ok = true;
    const void* take(size_t bytes) {
        if (!ok || off > size || bytes > size - off) {
            ok = false;
            return nullptr;
        }
        const void* p = base + off;
        off += bytes;
        return p;
    }
};

int fail_ck(int code, const char* what, const char* path) {
    char msg[512];
    snprintf(msg, sizeof msg, "checkpoint %s: %s", path ? path : "(null)", what);
    glmq::set_last_error(msg);
    fprintf(stderr, "[glm-cuda] %s\n", msg);
    return code;
}

}  // namespace

extern "C" int glm_cuda_load_checkpoint(const char* path, int device, int cache_cap) {
    if (!path || cache_cap < 1) return fail_ck(GLM_CUDA_ERR_ARG, "path must be non-NULL and cache_cap >= 1", path);
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail_ck(GLM_CUDA_ERR_ARG, "cannot open", path);
    struct stat stt {};
    if (fstat(fd, &stt) != 0 || stt.st_size < (off_t)kHeaderBytes) {
        close(fd);
        return fail_ck(GLM_CUDA_ERR_ARG, "too small for a header", path);
    }
    Mapped m;
    m.size = (size_t)stt.st_size;
    void* p = mmap(nullptr, m.size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return fail_ck(GLM_CUDA_ERR_ARG, "mmap failed", path);
    m.data = static_cast<const unsigned char*>(p);

    BinHeader h;
    memcpy(&h, m.data, sizeof h);
    // infer.c:375-385
    if (h.magic != kMagic) return fail_ck(GLM_CUDA_ERR_ARG, "bad magic", path);
    if (h.version < 4u || !(h.l0_flags & kFlagAllAttn))
        return fail_ck(GLM_CUDA_ERR_ARG, "needs format version 4 with every layer's attention", path);
    if (h.total_bytes != m.size) return fail_ck(GLM_CUDA_ERR_ARG, "size does not match the header", path);
    if (h.group_size == 0 || h.dim <= 0 || h.hidden_dim <= 0 || h.vocab_size <= 0 || h.n_layers < 2 ||
        h.moe_ffn_dim <= 0 || h.dim % (int)h.group_size || h.hidden_dim % (int)h.group_size ||
        h.q_lora_rank % (int)h.group_size || h.kv_lora_rank % (int)h.group_size ||
        h.moe_ffn_dim % (int)h.group_size || h.l0_qk_nope_dim % (int)h.group_size ||
        h.l0_head_k_dim != h.l0_qk_nope_dim + h.rope_dim)
        return fail_ck(GLM_CUDA_ERR_ARG, "inconsistent dimensions", path);

    GlmCudaModelDims d{};
    d.dim = h.dim;
    d.hidden_dim = h.hidden_dim;
    d.n_layers = h.n_layers;
    d.n_heads = h.n_heads;
    d.vocab_size = h.vocab_size;
    d.rope_dim = h.rope_dim;
    d.q_lora_rank = h.q_lora_rank;
    d.kv_lora_rank = h.kv_lora_rank;
    d.qk_nope_dim = h.l0_qk_nope_dim;
    d.head_k_dim = h.l0_head_k_dim;
    d.v_head_dim = h.l0_v_head_dim;
    d.n_routed_experts = h.n_routed_experts;
    d.n_experts_used = h.n_experts_used;
    d.group_size = (int32_t)h.group_size;
    d.moe_ffn_dim = h.moe_ffn_dim;
    d.cache_cap = cache_cap;
    if (int rc = glm_cuda_model_init(device, &d)) return rc;

    const size_t D = h.dim, H = h.hidden_dim, V = h.vocab_size, gs = h.group_size, NH = h.n_heads;
    const size_t QL = h.q_lora_rank, KL = h.kv_lora_rank, R = h.rope_dim, QN = h.l0_qk_nope_dim,
                 HK = h.l0_head_k_dim, VH = h.l0_v_head_dim, F = h.moe_ffn_dim, E = h.n_routed_experts;
    auto at = [&](uint64_t off, size_t bytes) -> const void* {
        return off <= m.size && bytes <= m.size - off ? m.data + off : nullptr;
    };
    // globals and layer-0 dense FFN at the header's offsets (infer.c:398-442)
    const void* g[12] = {at(h.off_norm, D * 4),          at(h.off_tok_q, V * D),
                         at(h.off_tok_s, V * D / gs * 4), at(h.off_out_q, V * D),
                         at(h.off_out_s, V * D / gs * 4), at(h.off_l0_ffn_norm, D * 4),
                         at(h.off_l0_ffn_gate_q, H * D),  at(h.off_l0_ffn_gate_s, H * D / gs * 4),
                         at(h.off_l0_ffn_up_q, H * D),    at(h.off_l0_ffn_up_s, H * D / gs * 4),
                         at(h.off_l0_ffn_down_q, D * H),  at(h.off_l0_ffn_down_s, D * H / gs * 4)};
    for (const void* q : g)
        if (!q) return fail_ck(GLM_CUDA_ERR_ARG, "global tensor out of bounds", path);
    if (int rc = glm_cuda_upload_model_globals(
            (const float*)g[0], (const int8_t*)g[1], (const float*)g[2], (const int8_t*)g[3], (const float*)g[4],
            (const float*)g[5], (const int8_t*)g[6], (const float*)g[7], (const int8_t*)g[8], (const float*)g[9],
            (const int8_t*)g[10], (const float*)g[11]))
        return rc;

    // one attention block: LayerAttnWeights order (model.h:46-62, infer.c:466-490)
    const size_t attn_bytes[15] = {D * 4,           QL * 4,           KL * 4,          QL * D,
                                   QL * D / gs * 4, NH * HK * QL,     NH * HK * QL / gs * 4,
                                   (KL + R) * D,    (KL + R) * D / gs * 4, NH * KL * QN,
                                   NH * KL * QN / gs * 4, NH * VH * KL, NH * VH * KL / gs * 4,
                                   D * NH * VH,     D * NH * VH / gs * 4};
    Cursor cur{m.data, m.size, (size_t)h.off_l0_ffn_down_s + D * H / gs * 4};
    for (size_t b : attn_bytes) cur.take(b);  // the layer-0 block of the v4 extension (infer.c:447-530)
    for (int l = 0; l < h.n_layers; ++l) {     // every layer's block (infer.c:533-626)
        const void* a[15];
        for (int i = 0; i < 15; ++i) a[i] = cur.take(attn_bytes[i]);
        if (!cur.ok) return fail_ck(GLM_CUDA_ERR_ARG, "attention block out of bounds", path);
        if (int rc = glm_cuda_upload_attn_layer(
                l, (const float*)a[0], (const float*)a[1], (const float*)a[2], (const int8_t*)a[3],
                (const float*)a[4], (const int8_t*)a[5], (const float*)a[6], (const int8_t*)a[7], (const float*)a[8],
                (const int8_t*)a[9], (const float*)a[10], (const int8_t*)a[11], (const float*)a[12],
                (const int8_t*)a[13], (const float*)a[14]))
            return rc;
    }
    // MoE layers 1..L-1: shared blocks, then routed blocks (infer.c:629-743)
    const size_t sh_bytes[9] = {D * 4, E * D * 4, E * 4, F * D, F * D / gs * 4, F * D, F * D / gs * 4, D * F,
                                D * F / gs * 4};
    const size_t rt_bytes[6] = {E * F * D, E * F * D / gs * 4, E * F * D, E * F * D / gs * 4, E * D * F,
                                E * D * F / gs * 4};
    const size_t sh_start = cur.off;
    size_t sh_total = 0;
    for (size_t b : sh_bytes) sh_total += b;
    Cursor rcur{m.data, m.size, sh_start + sh_total * (size_t)(h.n_layers - 1)};
    for (int l = 1; l < h.n_layers; ++l) {
        const void* s[9];
        const void* r[6];
        for (int i = 0; i < 9; ++i) s[i] = cur.take(sh_bytes[i]);
        for (int i = 0; i < 6; ++i) r[i] = rcur.take(rt_bytes[i]);
        if (!cur.ok || !rcur.ok) return fail_ck(GLM_CUDA_ERR_ARG, "MoE block out of bounds", path);
        if (int rc = glm_cuda_upload_moe_layer(l, (const float*)s[0], (const float*)s[1], (const float*)s[2],
                                               (const int8_t*)s[3], (const float*)s[4], (const int8_t*)s[5],
                                               (const float*)s[6], (const int8_t*)s[7], (const float*)s[8],
                                               (const int8_t*)r[0], (const float*)r[1], (const int8_t*)r[2],
                                               (const float*)r[3], (const int8_t*)r[4], (const float*)r[5]))
            return rc;
    }
    if (rcur.off != m.size) return fail_ck(GLM_CUDA_ERR_ARG, "trailing bytes after the routed experts", path);
    return 0;
}
