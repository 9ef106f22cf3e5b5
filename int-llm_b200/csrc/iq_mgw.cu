// iq_mgw.cu -- loads int-llm's native .mgw weight container into a device model.
//
// The .mgw file (llama_int.c:386-454) is a 64-byte header ("MGW\0", version 1,
// host-endian tag 0x01020304, tensor count, index and data offsets), a 64-byte
// config block (llama_config_t fields + lm_head_tied), 96-byte index entries
// (name, element count, data offset, ndims, shape) and 8-byte aligned int64
// Q16.48 data. mgw_load (llama_int.c:2344-2560) mmaps it and uses the tensors
// in place; here the file is mapped the same way, each tensor is checked as
// mgw_load checks it (bounds, names, the nine tensors of every layer) plus its
// element count against the config's shape, and handed to the model loaders
// (iq_model_load_globals / iq_model_load_layer), which copy each rank's rows to
// HBM and pack them. Errors are status returns, never exit().
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <cstring>
#include <string>
#include <vector>
#include "iq_common.cuh"

namespace {

struct MgwHeader {
    char magic[4];
    uint32_t version, endian_tag, num_tensors;
    uint64_t index_offset, data_offset;
    uint8_t reserved[32];
};
struct MgwConfig {
    int32_t hidden_dim, num_heads, num_kv_heads, head_dim, num_layers, intermediate_dim, vocab_size,
        max_seq_len, rope_theta, lm_head_tied, reserved[6];
};
struct MgwEntry {
    char name[64];
    uint64_t num_elements, data_offset;
    uint32_t ndims, shape[2], reserved;
};
static_assert(sizeof(MgwHeader) == 64, "mgw header is 64 bytes");
static_assert(sizeof(MgwConfig) == 64, "mgw config block is 64 bytes");
static_assert(sizeof(MgwEntry) == 96, "mgw index entry is 96 bytes");

const char *const kLayerSuffix[9] = {
    "input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
    "self_attn.v_proj.weight", "self_attn.o_proj.weight", "post_attention_layernorm.weight",
    "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"};

struct MgwMap {
    const uint8_t *base = nullptr;
    size_t size = 0;
    ~MgwMap() { if (base) munmap((void *)base, size); }
};

int mgw_map(const char *path, MgwMap *mm) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return IQ_ERR_ARG;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < (off_t)(sizeof(MgwHeader) + sizeof(MgwConfig))) {
        close(fd);
        return IQ_ERR_ARG;
    }
    void *p = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return IQ_ERR_ARG;
    mm->base = (const uint8_t *)p;
    mm->size = (size_t)sb.st_size;
    const MgwHeader *h = (const MgwHeader *)mm->base;
    if (memcmp(h->magic, "MGW\0", 4) != 0 || h->version != 1 || h->endian_tag != 0x01020304u) return IQ_ERR_ARG;
    const uint64_t iend = h->index_offset + (uint64_t)h->num_tensors * sizeof(MgwEntry);
    if (h->index_offset < sizeof(MgwHeader) + sizeof(MgwConfig) || iend > mm->size) return IQ_ERR_ARG;
    return IQ_OK;
}

void to_config(const MgwConfig &m, iq_config *c) {
    c->hidden_dim = m.hidden_dim;
    c->num_heads = m.num_heads;
    c->num_kv_heads = m.num_kv_heads;
    c->head_dim = m.head_dim;
    c->num_layers = m.num_layers;
    c->intermediate_dim = m.intermediate_dim;
    c->vocab_size = m.vocab_size;
    c->max_seq_len = m.max_seq_len;
    c->rope_theta = m.rope_theta;
}

}  // namespace

extern "C" {

IQ_API int iq_model_load_globals(iq_model *m, const int64_t *embed, const int64_t *final_norm,
                                 const int64_t *lm_head);
IQ_API int iq_model_load_layer(iq_model *m, int layer, const int64_t *const w[9]);
IQ_API int iq_model_config(const iq_model *m, iq_config *cfg);

IQ_API int iq_mgw_read_config(const char *path, iq_config *cfg, int *lm_head_tied) {
    if (!path || !cfg) return IQ_ERR_ARG;
    MgwMap mm;
    int rc = mgw_map(path, &mm);
    if (rc) return rc;
    const MgwConfig *mc = (const MgwConfig *)(mm.base + sizeof(MgwHeader));
    to_config(*mc, cfg);
    if (lm_head_tied) *lm_head_tied = mc->lm_head_tied;
    if (cfg->hidden_dim <= 0 || cfg->num_heads <= 0 || cfg->num_layers <= 0 || cfg->vocab_size <= 0)
        return IQ_ERR_ARG;  // llama_int.c:2411-2417
    return IQ_OK;
}

IQ_API int iq_model_load_mgw(iq_model *m, const char *path) {
    if (!m || !path) return IQ_ERR_ARG;
    MgwMap mm;
    int rc = mgw_map(path, &mm);
    if (rc) return rc;
    const MgwHeader *h = (const MgwHeader *)mm.base;
    const MgwConfig *mc = (const MgwConfig *)(mm.base + sizeof(MgwHeader));
    iq_config fc, c;
    to_config(*mc, &fc);
    if ((rc = iq_model_config(m, &c))) return rc;
    if (memcmp(&fc, &c, sizeof(c)) != 0) return IQ_ERR_ARG;  // the file describes another model
    const int L = c.num_layers, d = c.hidden_dim, kvd = c.num_kv_heads * c.head_dim, it = c.intermediate_dim;
    const uint64_t lsize[9] = {(uint64_t)d, (uint64_t)d * d, (uint64_t)kvd * d, (uint64_t)kvd * d,
                               (uint64_t)d * d, (uint64_t)d, (uint64_t)it * d, (uint64_t)it * d,
                               (uint64_t)d * it};
    const int64_t *embed = nullptr, *fnorm = nullptr, *lm = nullptr;
    std::vector<const int64_t *> lw((size_t)L * 9, nullptr);
    const MgwEntry *idx = (const MgwEntry *)(mm.base + h->index_offset);
    for (uint32_t i = 0; i < h->num_tensors; i++) {
        const MgwEntry &e = idx[i];
        char name[64];
        memcpy(name, e.name, 63);
        name[63] = '\0';
        const uint64_t bytes = e.num_elements * 8;
        if (e.num_elements > (1ull << 40) || e.data_offset % 8 || e.data_offset + bytes > mm.size)
            return IQ_ERR_ARG;  // llama_int.c:2447-2462
        const int64_t *p = (const int64_t *)(mm.base + e.data_offset);
        if (!strcmp(name, "model.embed_tokens.weight")) {
            if (e.num_elements != (uint64_t)c.vocab_size * d) return IQ_ERR_ARG;
            embed = p;
        } else if (!strcmp(name, "model.norm.weight")) {
            if (e.num_elements != (uint64_t)d) return IQ_ERR_ARG;
            fnorm = p;
        } else if (!strcmp(name, "lm_head.weight")) {
            if (e.num_elements != (uint64_t)c.vocab_size * d) return IQ_ERR_ARG;
            lm = p;
        } else {
            int l = -1, n = 0;
            if (sscanf(name, "model.layers.%d.%n", &l, &n) != 1 || n == 0 || l < 0 || l >= L) continue;
            for (int t = 0; t < 9; t++) {
                if (strcmp(name + n, kLayerSuffix[t])) continue;
                if (e.num_elements != lsize[t] || lw[(size_t)l * 9 + t]) return IQ_ERR_ARG;
                lw[(size_t)l * 9 + t] = p;
            }
        }
    }
    if (mc->lm_head_tied) lm = embed;  // llama_int.c:2525-2528
    if (!embed || !fnorm || !lm) return IQ_ERR_ARG;
    for (const int64_t *p : lw)
        if (!p) return IQ_ERR_ARG;   // every layer needs its nine tensors (llama_int.c:2538-2546)
    if ((rc = iq_model_load_globals(m, embed, fnorm, lm))) return rc;
    for (int l = 0; l < L; l++)
        if ((rc = iq_model_load_layer(m, l, lw.data() + (size_t)l * 9))) return rc;
    return IQ_OK;
}

}  // extern "C"
