// step_schedule.h - host-side plan of the persistent decode-step kernel
// (decode_step.cuh): which weight rows every contraction CTA owns, and the
// order, size and shared-memory placement of every bulk copy it streams.
//
// Plain C++ (no CUDA): the kernel reads the copy list the host builds here,
// and tests/test_step_schedule.py compiles this header on the CPU to check
// that live copies never overlap in the ring and that every matrix row has
// exactly one owner.
//
// Per contraction CTA j of n, one decode step streams, in the order the
// kernel consumes them:
//   for every layer:  [attn_norm gains][its q|k|v blocks]      (if it owns any)
//                     [its o blocks]                            (if any)
//                     [ffn_norm gains][its gate|up block pairs] (if any)
//                     [its down blocks]                         (if any)
//   then              [out_norm gains][its lm_head blocks, in chunks]
// Matrices are split into balanced contiguous block ranges,
// [j * NB / n, (j + 1) * NB / n). o and down split the same 2048 rows the
// same way, so a CTA owns the same residual rows in both.
//
// The copies go through a byte ring: copy i lands at ring_off, right after
// copy i-1, or at 0 when it would run past the end. Before issuing copy i
// the producer waits until the consumer has released every copy before
// `need` (copy i overlaps none of copies need .. i-1, and at most kSlots
// copies are in flight, one mbarrier pair each).
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#ifdef __CUDACC__
#define BNN_STEP_HD __host__ __device__
#else
#define BNN_STEP_HD
#endif

namespace bnn {
namespace step {

constexpr uint32_t kSlots = 16;          // copies in flight per CTA (mbarrier pairs)
constexpr uint32_t kLmChunkBlocks = 16;  // lm_head blocks per copy (at most)

struct Copy {
    uint64_t src;       // device address
    uint32_t bytes;
    uint32_t ring_off;  // byte offset in the CTA's ring
    uint32_t need;      // copies released before this one may be issued
    uint32_t blocks;    // weight blocks in the copy (0: a gains vector)
};

BNN_STEP_HD inline void split(uint32_t j, uint32_t n, uint32_t nb, uint32_t* b0, uint32_t* b1) {
    *b0 = (uint32_t)((uint64_t)j * nb / n);
    *b1 = (uint32_t)((uint64_t)(j + 1) * nb / n);
}

struct LayerSrc {
    uint64_t qkv, o, gu, down;     // packed block arrays
    uint64_t attn_norm, ffn_norm;  // gains [C]
};

struct ScheduleShape {
    uint32_t layers, hidden, ffn, qkv_rows, vocab;
    uint32_t n_gemv;      // contraction CTAs
    uint32_t ring_bytes;  // ring capacity per CTA
};

// Block bytes of a packed W1 matrix with `groups` 128-wide groups.
inline uint32_t sched_block_bytes(uint32_t groups) { return groups * 144u; }

// Appends copy (src, bytes) to `out`, placing it in the ring. Returns false
// when a single copy does not fit the ring.
inline bool place(std::vector<Copy>& out, uint64_t src, uint32_t bytes, uint32_t blocks, uint32_t ring) {
    if (bytes == 0 || bytes > ring || bytes % 16u)
        return false;
    Copy c{src, bytes, 0, 0, blocks};
    const size_t i = out.size();
    if (i > 0) {
        const Copy& p = out.back();
        uint32_t off = (p.ring_off + p.bytes + 127u) & ~127u;
        if ((uint64_t)off + bytes > ring)
            off = 0;
        c.ring_off = off;
        c.need = p.need;
    }
    // the oldest copy that must stay live: none of need .. i-1 may overlap
    for (size_t k = i; k-- > c.need;) {
        const Copy& q = out[k];
        const bool overlap = q.ring_off < c.ring_off + bytes && c.ring_off < q.ring_off + q.bytes;
        if (overlap) {
            c.need = (uint32_t)(k + 1);
            break;
        }
    }
    if (i >= kSlots && c.need < i - kSlots + 1)
        c.need = (uint32_t)(i - kSlots + 1);
    out.push_back(c);
    return true;
}

// The copy list of contraction CTA j. Returns false if some copy does not
// fit the ring.
inline bool build_schedule(const ScheduleShape& s, const std::vector<LayerSrc>& layers, uint64_t lm_head,
                           uint64_t out_norm, uint32_t j, std::vector<Copy>* out) {
    out->clear();
    const uint32_t gc = s.hidden / 128u, gf = s.ffn / 128u;
    const uint32_t bbc = sched_block_bytes(gc), bbf = sched_block_bytes(gf);
    const uint32_t nb_qkv = s.qkv_rows / 8u, nb_c = s.hidden / 8u, np_gu = s.ffn / 8u;
    const uint32_t nb_v = (s.vocab + 7u) / 8u;
    uint32_t q0, q1, o0, o1, p0, p1, v0, v1;
    split(j, s.n_gemv, nb_qkv, &q0, &q1);
    split(j, s.n_gemv, nb_c, &o0, &o1);
    split(j, s.n_gemv, np_gu, &p0, &p1);
    split(j, s.n_gemv, nb_v, &v0, &v1);
    const uint32_t R = s.ring_bytes;
    for (uint32_t l = 0; l < s.layers; ++l) {
        const LayerSrc& L = layers[l];
        if (q1 > q0 && !(place(*out, L.attn_norm, s.hidden * 4u, 0, R) &&
                         place(*out, L.qkv + (uint64_t)q0 * bbc, (q1 - q0) * bbc, q1 - q0, R)))
            return false;
        if (o1 > o0 && !place(*out, L.o + (uint64_t)o0 * bbc, (o1 - o0) * bbc, o1 - o0, R))
            return false;
        if (p1 > p0 && !(place(*out, L.ffn_norm, s.hidden * 4u, 0, R) &&
                         place(*out, L.gu + (uint64_t)2u * p0 * bbc, 2u * (p1 - p0) * bbc, 2u * (p1 - p0), R)))
            return false;
        if (o1 > o0 && !place(*out, L.down + (uint64_t)o0 * bbf, (o1 - o0) * bbf, o1 - o0, R))
            return false;
    }
    if (v1 > v0) {
        if (!place(*out, out_norm, s.hidden * 4u, 0, R))
            return false;
        for (uint32_t b = v0; b < v1; b += kLmChunkBlocks) {
            const uint32_t nb = v1 - b < kLmChunkBlocks ? v1 - b : kLmChunkBlocks;
            if (!place(*out, lm_head + (uint64_t)b * bbc, nb * bbc, nb, R))
                return false;
        }
    }
    return true;
}

}  // namespace step
}  // namespace bnn
