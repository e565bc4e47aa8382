// synth.cpp - seeded synthetic models in the engine's binding layout.
//
// Builds a nya_llm_context exactly as the engine's GGUF loader binds a dense
// LLaMA model (backend/core/llm_gguf.c:1013-1118: token_embd, output_norm,
// output, blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,
// ffn_gate,ffn_down,ffn_up}; cache_offset = layer * kv_dim) but with random
// tensor contents, so the engine's CPU path and this provider can run the
// same bytes. Contents are a pure function of (seed, tensor index, block
// index): every block is generated from its own counter, so any row range
// can be produced independently and in parallel.
//
// Value distributions (per GGUF block):
//   Q4_K: d, dmin = fp16(|N(0,1)| * 0.01); 8 scales and 8 mins uniform in
//         [0,63], packed like test_architectures.c:254-258; nibbles uniform.
//   Q6_K: 6-bit quants uniform; 16 int8 scales uniform in [0,63];
//         d = fp16(|N(0,1)| * 0.01).
//   Q8_0: 32 int8 uniform in [-127,127]; d = fp16(|N(0,1)| * 0.01).
//   F32/F16/BF16 matrices: N(0,1) * 0.02. Norm vectors per norm_mode.
#include "fyodor_b200.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>
#include <chrono>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace {

inline uint64_t splitmix(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

struct Rng {
    uint64_t state;
    Rng(uint64_t seed, uint64_t stream, uint64_t block)
        : state(splitmix(seed ^ splitmix(stream * 0x632BE59BD9B4E019ull + 1) ^ splitmix(block + 0x1234567ull))) {}
    uint64_t next() { state = splitmix(state); return state; }
    double uniform() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
    double normal()
    {
        double u1 = uniform(), u2 = uniform();
        if (u1 < 1e-300) u1 = 1e-300;
        return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
    }
};

// float -> binary16 bits, round to nearest even (same rule as the engine's
// nya_llm_round_f16, backend/core/llm_quant.c:46-67).
uint16_t half_bits(float value)
{
    uint32_t bits;
    std::memcpy(&bits, &value, 4);
    uint32_t sign = (bits >> 16) & 0x8000u, mag = bits & 0x7fffffffu, r;
    if (mag >= 0x7f800000u) r = mag == 0x7f800000u ? 0x7c00u : 0x7e00u;
    else if (mag >= 0x477ff000u) r = 0x7c00u;
    else if (mag < 0x33000000u) r = 0;
    else {
        uint32_t e = mag >> 23, shift = e < 113u ? 126u - e : 13u;
        uint32_t m = (mag & 0x7fffffu) | (e < 113u ? 0x800000u : 0u);
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        r = e < 113u ? q : ((e - 112u) << 10) + q;
    }
    return (uint16_t)(sign | r);
}

void put16(unsigned char *p, uint16_t v) { p[0] = (unsigned char)v; p[1] = (unsigned char)(v >> 8); }

size_t block_values(uint32_t type)
{
    switch (type) {
    case 12: case 14: return 256;
    case 2: case 8: return 32;
    default: return 1;
    }
}
size_t block_bytes(uint32_t type)
{
    switch (type) {
    case 0: return 4;
    case 1: case 30: return 2;
    case 2: return 18;
    case 8: return 34;
    case 12: return 144;
    case 14: return 210;
    default: return 0;
    }
}

float half_value(uint16_t h)
{
    uint32_t e = (h >> 10) & 31u, f = h & 1023u;
    float v = e ? std::ldexp((float)(1024u + f), (int)e - 25) : std::ldexp((float)f, -24);
    return (h & 0x8000u) ? -v : v;
}

void fill_block(unsigned char *p, uint32_t type, Rng &r, int centered)
{
    switch (type) {
    case 12: {
        const uint16_t dh = half_bits((float)(std::fabs(r.normal()) * 0.01));
        const uint16_t mh = half_bits((float)(std::fabs(r.normal()) * 0.01));
        put16(p, dh);
        put16(p + 2, mh);
        unsigned sc[8], mn[8];
        for (int g = 0; g < 8; ++g) { sc[g] = (unsigned)(r.next() & 63); mn[g] = (unsigned)(r.next() & 63); }
        if (centered) {
            // mean of d*sc*q - dmin*m over uniform nibbles is d*sc*7.5 - dmin*m
            const float d = half_value(dh), dm = half_value(mh);
            for (int g = 0; g < 8; ++g) {
                double m = dm > 0 ? std::nearbyint(7.5 * d * sc[g] / dm) : 0.0;
                mn[g] = (unsigned)(m < 0 ? 0 : m > 63 ? 63 : m);
            }
        }
        for (int g = 0; g < 4; ++g) {
            p[4 + g] = (unsigned char)(sc[g] | ((sc[g + 4] >> 4) << 6));
            p[8 + g] = (unsigned char)(mn[g] | ((mn[g + 4] >> 4) << 6));
            p[12 + g] = (unsigned char)((sc[g + 4] & 15) | ((mn[g + 4] & 15) << 4));
        }
        for (int i = 0; i < 128; i += 8) { uint64_t w = r.next(); std::memcpy(p + 16 + i, &w, 8); }
        break;
    }
    case 14: {
        for (int i = 0; i < 192; i += 8) { uint64_t w = r.next(); std::memcpy(p + i, &w, 8); }
        for (int g = 0; g < 16; ++g) p[192 + g] = (unsigned char)(r.next() & 63);
        put16(p + 208, half_bits((float)(std::fabs(r.normal()) * 0.01)));
        break;
    }
    case 8: {
        put16(p, half_bits((float)(std::fabs(r.normal()) * 0.01)));
        for (int i = 0; i < 32; ++i) p[2 + i] = (unsigned char)(signed char)((int)(r.next() % 255) - 127);
        break;
    }
    case 2: {
        put16(p, half_bits((float)(std::fabs(r.normal()) * 0.01)));
        for (int i = 0; i < 16; ++i) p[2 + i] = (unsigned char)r.next();
        break;
    }
    case 0: { float v = (float)(r.normal() * 0.02); std::memcpy(p, &v, 4); break; }
    case 1: put16(p, half_bits((float)(r.normal() * 0.02))); break;
    case 30: {
        float v = (float)(r.normal() * 0.02);
        uint32_t b; std::memcpy(&b, &v, 4);
        put16(p, (uint16_t)(b >> 16));
        break;
    }
    default: break;
    }
}

// Fill rows [r0, r1) of a matrix; block b of row r uses counter r*nblk+b.
void fill_rows(unsigned char *data, size_t r0, size_t r1, size_t columns, uint32_t type, uint64_t seed, uint64_t stream,
    int centered)
{
    size_t nb = columns / block_values(type), bb = block_bytes(type), row_bytes = nb * bb;
    if (block_values(type) == 1) {
        // scalar types: one generator per row
        for (size_t r = r0; r < r1; ++r) {
            Rng g(seed, stream, r);
            for (size_t c = 0; c < columns; ++c) fill_block(data + r * row_bytes + c * bb, type, g, centered);
        }
        return;
    }
    for (size_t r = r0; r < r1; ++r)
        for (size_t b = 0; b < nb; ++b) {
            Rng g(seed, stream, r * nb + b);
            fill_block(data + r * row_bytes + b * bb, type, g, centered);
        }
}

void fill_parallel(unsigned char *data, size_t rows, size_t columns, uint32_t type, uint64_t seed, uint64_t stream, int threads,
    int centered)
{
    if (threads <= 1 || rows < 64) { fill_rows(data, 0, rows, columns, type, seed, stream, centered); return; }
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        size_t a = rows * t / threads, b = rows * (t + 1) / threads;
        pool.emplace_back(fill_rows, data, a, b, columns, type, seed, stream, centered);
    }
    for (auto &th : pool) th.join();
}

struct SynthOwner {  // stored in mapping.data so fyb_synth_free can release everything
    unsigned char *arena;
};

constexpr uint64_t SYNTH_MAGIC = 0x4659425359544831ull;  // "FYBSYTH1"

// Digest of everything that determines a model's bytes (a shared file made
// for another configuration is not used).
uint64_t config_digest(const fyb_synth_config &c, size_t total)
{
    uint64_t h = splitmix(total);
    const uint64_t f[] = {c.layers, c.embedding, c.heads, c.kv_heads, c.feed_forward, c.vocabulary, c.context,
                          c.matrix_type, c.embed_type, c.output_type, (uint64_t)(uint32_t)c.norm_mode,
                          (uint64_t)(uint32_t)c.centered, c.seed};
    for (uint64_t v : f) h = splitmix(h ^ v);
    return h;
}

}  // namespace

extern "C" void fyb_synth_fill(void *data, size_t rows, size_t columns, uint32_t type, uint64_t seed, uint64_t stream_id)
{
    fill_parallel((unsigned char *)data, rows, columns, type, seed, stream_id, 1, 0);
}

extern "C" nya_llm_context *fyb_synth_create(const fyb_synth_config *cfg)
{
    if (!cfg || !cfg->layers || !cfg->embedding || !cfg->heads || !cfg->kv_heads || cfg->heads % cfg->kv_heads ||
        cfg->embedding % cfg->heads || !cfg->feed_forward || !cfg->vocabulary || !cfg->context || cfg->layers > 256)
        return nullptr;
    const uint32_t d = cfg->embedding, hd = d / cfg->heads, kvd = hd * cfg->kv_heads, ffn = cfg->feed_forward;
    const uint32_t mt = cfg->matrix_type, et = cfg->embed_type, ot = cfg->output_type;
    auto aligned_ok = [](uint32_t type, uint32_t cols) { return block_bytes(type) && cols % block_values(type) == 0; };
    if (!aligned_ok(mt, d) || !aligned_ok(mt, ffn) || !aligned_ok(et, d) || !aligned_ok(ot, d)) return nullptr;
    int threads = cfg->threads > 0 ? cfg->threads : (int)std::thread::hardware_concurrency();
    if (threads <= 0) threads = 1;

    nya_llm_context *c = (nya_llm_context *)std::calloc(1, sizeof(nya_llm_context));
    if (!c) return nullptr;
    const size_t ntensors = 3 + (size_t)cfg->layers * 9;
    c->tensors = (nya_llm_tensor *)std::calloc(ntensors, sizeof(nya_llm_tensor));
    c->layers = (nya_llm_layer *)std::calloc(cfg->layers, sizeof(nya_llm_layer));
    if (!c->tensors || !c->layers) { fyb_synth_free(c); return nullptr; }
    c->tensor_count = ntensors;

    struct Spec { const char *fmt; uint32_t type, cols, rows; int layer; };
    std::vector<Spec> specs;
    specs.push_back({"token_embd.weight", et, d, cfg->vocabulary, -1});
    specs.push_back({"output_norm.weight", 0, d, 1, -1});
    specs.push_back({"output.weight", ot, d, cfg->vocabulary, -1});
    for (uint32_t l = 0; l < cfg->layers; ++l) {
        specs.push_back({"blk.%u.attn_norm.weight", 0, d, 1, (int)l});
        specs.push_back({"blk.%u.attn_q.weight", mt, d, d, (int)l});
        specs.push_back({"blk.%u.attn_k.weight", mt, d, kvd, (int)l});
        specs.push_back({"blk.%u.attn_v.weight", mt, d, kvd, (int)l});
        specs.push_back({"blk.%u.attn_output.weight", mt, d, d, (int)l});
        specs.push_back({"blk.%u.ffn_norm.weight", 0, d, 1, (int)l});
        specs.push_back({"blk.%u.ffn_gate.weight", mt, d, ffn, (int)l});
        specs.push_back({"blk.%u.ffn_down.weight", mt, ffn, d, (int)l});
        specs.push_back({"blk.%u.ffn_up.weight", mt, d, ffn, (int)l});
    }
    size_t total = 0;
    std::vector<size_t> offsets(specs.size());
    for (size_t i = 0; i < specs.size(); ++i) {
        offsets[i] = total;
        size_t bytes = (size_t)specs[i].rows * (specs[i].cols / block_values(specs[i].type)) * block_bytes(specs[i].type);
        total += (bytes + 255) / 256 * 256;
    }
    unsigned char *arena = nullptr;
    bool fill = true;
    if (cfg->path) {
        // header page: magic, configuration digest, byte count, complete flag
        const uint64_t digest = config_digest(*cfg, total);
        const size_t head = 4096, bytes = head + total;
        int fd = ::open(cfg->path, O_RDWR | O_CREAT | O_EXCL, 0600);
        const bool creator = fd >= 0;
        if (!creator) fd = ::open(cfg->path, O_RDONLY);
        if (fd < 0) { fyb_synth_free(c); return nullptr; }
        if (creator && ::ftruncate(fd, (off_t)bytes) != 0) { ::close(fd); ::unlink(cfg->path); fyb_synth_free(c); return nullptr; }
        if (!creator) {  // wait (bounded) for the creator to size and complete it
            bool ready = false;
            for (int i = 0; i < 6000 && !ready; ++i) {
                struct stat st;
                if (::fstat(fd, &st) == 0 && (size_t)st.st_size == bytes) {
                    uint64_t hdr[4] = {0, 0, 0, 0};
                    const bool read = ::pread(fd, hdr, sizeof(hdr), 0) == (ssize_t)sizeof(hdr);
                    if (read && hdr[3] == 1 && (hdr[0] != SYNTH_MAGIC || hdr[1] != digest || hdr[2] != total))
                        break;  // complete, but made for another configuration
                    ready = read && hdr[0] == SYNTH_MAGIC && hdr[1] == digest && hdr[2] == total && hdr[3] == 1;
                }
                else {
                    struct stat st2;
                    if (::fstat(fd, &st2) == 0 && (size_t)st2.st_size != bytes && st2.st_size != 0) {
                        uint64_t hdr[4] = {0, 0, 0, 0};
                        if (::pread(fd, hdr, sizeof(hdr), 0) == (ssize_t)sizeof(hdr) && hdr[3] == 1) break;
                    }
                }
                if (!ready) std::this_thread::sleep_for(std::chrono::milliseconds(100));
            }
            if (!ready) { ::close(fd); fyb_synth_free(c); return nullptr; }
        }
        void *m = ::mmap(nullptr, bytes, creator ? PROT_READ | PROT_WRITE : PROT_READ, MAP_SHARED, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED) { if (creator) ::unlink(cfg->path); fyb_synth_free(c); return nullptr; }
        arena = (unsigned char *)m + head;
        c->mapping.data = (unsigned char *)m;
        c->mapping.size = bytes;
        c->mapping.mapping_handle = 1;  // a shared-file mapping: fyb_synth_free unmaps it
        fill = creator;
    } else {
        arena = (unsigned char *)std::aligned_alloc(256, total ? total : 256);
        if (!arena) { fyb_synth_free(c); return nullptr; }
        c->mapping.data = arena;
        c->mapping.size = total;
    }
    for (size_t i = 0; i < specs.size(); ++i) {
        nya_llm_tensor *t = &c->tensors[i];
        const Spec &s = specs[i];
        if (s.layer >= 0) std::snprintf(t->name, sizeof(t->name), s.fmt, (unsigned)s.layer);
        else std::snprintf(t->name, sizeof(t->name), "%s", s.fmt);
        t->type = s.type;
        t->dimension_count = s.rows == 1 ? 1 : 2;
        t->dimensions[0] = s.cols;
        t->dimensions[1] = s.rows;
        t->relative_offset = offsets[i];
        t->data = arena + offsets[i];
        t->data_size = (size_t)s.rows * (s.cols / block_values(s.type)) * block_bytes(s.type);
        t->bound = 1;
        unsigned char *dst = arena + offsets[i];
        if (!fill) continue;
        if (s.rows == 1) {  // norm vector
            Rng g(cfg->seed, i, 0);
            for (uint32_t k = 0; k < s.cols; ++k) {
                float v = cfg->norm_mode == 0 ? 1.0f : cfg->norm_mode == 1 ? (float)(1.0 + 0.01 * g.normal()) : (float)g.normal();
                std::memcpy(dst + 4 * k, &v, 4);
            }
        } else {
            fill_parallel(dst, s.rows, s.cols, s.type, cfg->seed, i, threads, cfg->centered);
        }
    }
    if (cfg->path && fill) {  // the file is complete: later processes may map it
        uint64_t *hdr = (uint64_t *)c->mapping.data;
        hdr[0] = SYNTH_MAGIC; hdr[1] = config_digest(*cfg, total); hdr[2] = total;
        __atomic_store_n(&hdr[3], (uint64_t)1, __ATOMIC_RELEASE);
    }
    c->token_embedding = &c->tensors[0];
    c->output_norm = &c->tensors[1];
    c->output = &c->tensors[2];
    for (uint32_t l = 0; l < cfg->layers; ++l) {
        nya_llm_layer *w = &c->layers[l];
        nya_llm_tensor *b = &c->tensors[3 + (size_t)l * 9];
        w->attention_norm = b + 0; w->query = b + 1; w->key = b + 2; w->value = b + 3;
        w->attention_output = b + 4; w->feed_forward_norm = b + 5; w->feed_forward_gate = b + 6;
        w->feed_forward_down = b + 7; w->feed_forward_up = b + 8;
        w->head_count = cfg->heads; w->kv_head_count = cfg->kv_heads; w->head_dimension = hd;
        w->hidden_length = ffn; w->kv_source = l; w->cache_offset = (size_t)l * kvd;
    }
    c->tokenizer.vocabulary_size = cfg->vocabulary;
    c->embedding_length = d;
    c->feed_forward_length = ffn;
    c->block_count = cfg->layers;
    c->head_count = cfg->heads;
    c->key_value_head_count = cfg->kv_heads;
    c->context_length = cfg->context;
    c->rope_dimension_count = hd;
    c->norm_epsilon = cfg->epsilon > 0 ? cfg->epsilon : 1e-5f;
    c->rope_frequency_base = cfg->rope_base > 0 ? cfg->rope_base : 500000.0f;
    c->head_dimension = hd;
    c->sliding_head_dimension = hd;
    c->cache_width = (size_t)cfg->layers * kvd;
    c->maximum_query_length = d;
    c->maximum_hidden_length = ffn;
    c->heads_count = 1; c->kv_heads_count = 1; c->hidden_count = 1;
    c->layer_heads[0] = cfg->heads; c->layer_kv_heads[0] = cfg->kv_heads; c->layer_hidden[0] = ffn;
    c->value_dimension = hd;
    c->tensor_alignment = 256;
    return c;
}

extern "C" void fyb_synth_free(nya_llm_context *c)
{
    if (!c) return;
    if (c->mapping.mapping_handle == 1) ::munmap(c->mapping.data, c->mapping.size);
    else std::free(c->mapping.data);
    std::free(c->tensors);
    std::free(c->layers);
    std::free(c);
}
