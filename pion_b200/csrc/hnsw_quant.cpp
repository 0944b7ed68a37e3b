// Host side of the block-quantised HNSW formats (the reference builds them on the host in
// compact_vectors): one slot per node in the graph's slot order, plus TurboQuant's QJL
// rows by node.
//   quantize_fp32_to_block_int4 / _int3 / _int2   src/vector/kernels.mojo:1116-1842
//   qjl_compute_signs, wht_fp32_1536              kernels.mojo:981-1019, 1685-1714
//   the residual of the INT3 codes, rows by node  src/vector/hnsw.mojo:3138-3230
//   the QJL sign flips (LCG seeded 42)            src/vector/hnsw.mojo:497-509
// Float arithmetic in the reference's order (two roundings per a*b+c: the ISA target
// x86-64-v2 has no FMA); f16 scales rounded to nearest even.
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "hnsw_host.h"

namespace pion {
namespace hnsw {

namespace {

constexpr int kDim = 1536;
constexpr int kBlocks = 48;

uint16_t to_half(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ex = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (ex == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    const int e = (int)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

float from_half(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t x;
    if (ex == 0) {
        if (man == 0) {
            x = sign;
        } else {
            int e = -1;
            uint32_t m = man;
            do {
                ++e;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (ex == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((ex - 15 + 127) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

// Int(q + 0.5) for q >= 0, Int(q - 0.5) below: half away from zero, then truncation.
inline int round_away(float q) {
    volatile float t = q >= 0.0f ? q + 0.5f : q - 0.5f;
    return (int)t;
}

inline float mul(float a, float b) {
    volatile float r = a * b;
    return r;
}

inline float add(float a, float b) {
    volatile float r = a + b;
    return r;
}

// l2_normalize_fp32 (src/vector/kernels.mojo:318-357): four lane sums combined
// (s0 + s2) + (s1 + s3), the tail in order, inv = 1/sqrt; a zero row passes through.
void l2_normalize(const float* x, float* y) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < kDim; ++d) s[d & 3] = add(s[d & 3], mul(x[d], x[d]));
    const float ns = add(add(s[0], s[2]), add(s[1], s[3]));
    if (ns <= 0.0f) {
        std::memcpy(y, x, kDim * sizeof(float));
        return;
    }
    const float inv = 1.0f / std::sqrt(ns);
    for (int d = 0; d < kDim; ++d) y[d] = mul(x[d], inv);
}

void block_slot(int kind, const float* src, int8_t* dst) {
    float recon = 0.0f;
    int off = 4;
    const float qmax = kind == kQuantPolar ? 7.0f : kind == kQuantNano ? 1.5f : 3.0f;
    for (int b = 0; b < kBlocks; ++b) {
        const float* x = src + b * 32;
        float absmax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            const float av = x[i] >= 0 ? x[i] : -x[i];
            if (av > absmax) absmax = av;
        }
        const float scale = absmax > 0 ? absmax / qmax : 1.0f;
        const float inv = 1.0f / scale;
        int q[32];
        uint16_t hs;
        if (kind == kQuantNano) {
            const float stored = mul(scale, 0.5f);
            hs = to_half(stored);
            for (int i = 0; i < 32; ++i) {
                int v = round_away(add(mul(x[i], inv), 1.5f));
                v = v > 3 ? 3 : (v < 0 ? 0 : v);
                q[i] = v;
                const float r = mul((float)(v * 2 - 3), stored);
                recon = add(recon, mul(r, r));
            }
        } else {
            hs = to_half(scale);
            const int lo = kind == kQuantPolar ? -8 : -4, hi = kind == kQuantPolar ? 7 : 3;
            for (int i = 0; i < 32; ++i) {
                int v = round_away(mul(x[i], inv));
                v = v > hi ? hi : (v < lo ? lo : v);
                q[i] = v;
                const float r = mul((float)v, scale);
                recon = add(recon, mul(r, r));
            }
        }
        std::memcpy(dst + off, &hs, 2);
        off += 2;
        uint8_t* d = reinterpret_cast<uint8_t*>(dst) + off;
        if (kind == kQuantPolar) {
            for (int i = 0; i < 16; ++i) d[i] = (uint8_t)(((q[i + 16] + 8) << 4) | (q[i] + 8));
            off += 16;
        } else if (kind == kQuantNano) {
            for (int g = 0; g < 8; ++g)
                d[g] = (uint8_t)(q[4 * g] | (q[4 * g + 1] << 2) | (q[4 * g + 2] << 4) |
                                 (q[4 * g + 3] << 6));
            off += 8;
        } else {
            for (int g = 0; g < 4; ++g) {
                int v[8];
                for (int i = 0; i < 8; ++i) v[i] = q[8 * g + i] + 4;
                uint8_t* o = d + 3 * g;
                o[0] = (uint8_t)(v[0] | (v[1] << 3) | ((v[2] & 3) << 6));
                o[1] = (uint8_t)((v[2] >> 2) | (v[3] << 1) | (v[4] << 4) | ((v[5] & 1) << 7));
                o[2] = (uint8_t)((v[5] >> 1) | (v[6] << 2) | (v[7] << 5));
            }
            off += 12;
        }
    }
    std::memcpy(dst, &recon, 4);
}

void wht512(float* d) {
    for (int h = 1; h < 512; h *= 2)
        for (int i = 0; i < 512; i += 2 * h)
            for (int j = 0; j < h; ++j) {
                const float x = d[i + j], y = d[i + j + h];
                d[i + j] = add(x, y);
                d[i + j + h] = add(x, -y);
            }
    const float nv = 0.044194173824159216f;
    for (int i = 0; i < 512; ++i) d[i] = mul(d[i], nv);
}

float qjl_row(const float* src, const int8_t* slot, const uint64_t* rs, uint64_t* dst) {
    float t[kDim];
    float n2 = 0.0f;
    for (int b = 0; b < kBlocks; ++b) {
        uint16_t hs;
        std::memcpy(&hs, slot + 4 + b * 14, 2);
        const float sv = from_half(hs);
        const uint8_t* d = reinterpret_cast<const uint8_t*>(slot) + 4 + b * 14 + 2;
        for (int g = 0; g < 4; ++g) {
            const uint64_t u = (uint64_t)d[3 * g] | ((uint64_t)d[3 * g + 1] << 8) |
                               ((uint64_t)d[3 * g + 2] << 16);
            for (int k = 0; k < 8; ++k) {
                const int i = b * 32 + 8 * g + k;
                const float r = add(src[i], -mul((float)((int)((u >> (3 * k)) & 7) - 4), sv));
                const float s = ((rs[i >> 6] >> (i & 63)) & 1ull) ? 1.0f : -1.0f;
                t[i] = mul(r, s);
                n2 = add(n2, mul(r, r));
            }
        }
    }
    wht512(t);
    wht512(t + 512);
    wht512(t + 1024);
    for (int w = 0; w < 24; ++w) {
        uint64_t bits = 0;
        for (int b = 0; b < 64; ++b)
            if (t[w * 64 + b] > 0) bits |= 1ull << b;
        dst[w] = bits;
    }
    return n2;
}

}  // namespace

int64_t quant_stride(int kind) {
    return kind == kQuantPolar ? 868 : kind == kQuantNano ? 484 : 676;
}

void qjl_random_signs(uint64_t* out24) {
    uint64_t s = 42;
    for (int w = 0; w < 24; ++w) {
        uint64_t bits = 0;
        for (int b = 0; b < 64; ++b) {
            s = s * 6364136223846793005ull + 1442695040888963407ull;
            if ((s >> 33) & 1ull) bits |= 1ull << b;
        }
        out24[w] = bits;
    }
}

int quantize(const Graph& g, const float* rows, int kind, QuantBuffers& out, std::string& why) {
    if (kind < kQuantPolar || kind > kQuantTurbo) {
        why = "unknown kind";
        return -1;
    }
    if (g.dim != kDim || g.n <= 0 || g.node_slot.size() != (size_t)g.n) {
        why = "the graph has no 1536-dim layout";
        return -3;
    }
    const int64_t n = g.n, stride = quant_stride(kind);
    out = QuantBuffers{};
    out.kind = kind;
    out.stride = stride;
    out.compact.assign((size_t)(n * stride), 0);
    out.rerank.resize((size_t)n * kDim);
    if (kind == kQuantTurbo) {
        out.qjl.assign((size_t)n * 24, 0ull);
        out.qjl_res_norms.assign((size_t)n, 0.0f);
        out.random_signs.resize(24);
        qjl_random_signs(out.random_signs.data());
    }
    for (int64_t i = 0; i < n; ++i)
        if (g.node_slot[i] >= (uint64_t)n) {
            why = "node_slot out of range";
            return -3;
        }
    // every node is independent: contiguous node ranges on the host threads
    auto work = [&](int64_t lo, int64_t hi) {
        std::vector<float> x(kDim);
        for (int64_t i = lo; i < hi; ++i) {
            const float* r = rows + i * kDim;
            if (g.metric == 1) {  // the stored rows of a COSINE index are normalised
                l2_normalize(r, x.data());
            } else {
                std::memcpy(x.data(), r, kDim * sizeof(float));
            }
            std::memcpy(out.rerank.data() + (size_t)i * kDim, x.data(), kDim * sizeof(float));
            int8_t* slot = out.compact.data() + (size_t)g.node_slot[i] * stride;
            block_slot(kind, x.data(), slot);
            if (kind == kQuantTurbo)
                out.qjl_res_norms[i] = qjl_row(x.data(), slot, out.random_signs.data(),
                                               out.qjl.data() + (size_t)i * 24);
        }
    };
    int64_t threads = (int64_t)std::thread::hardware_concurrency();
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    if (threads > n / 256 + 1) threads = n / 256 + 1;
    std::vector<std::thread> pool;
    for (int64_t t = 1; t < threads; ++t)
        pool.emplace_back(work, n * t / threads, n * (t + 1) / threads);
    work(0, n / threads);
    for (auto& th : pool) th.join();
    return 0;
}

}  // namespace hnsw
}  // namespace pion
