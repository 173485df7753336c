// decode_common.cuh -- work schedule and chunk merge shared by the decode kernels
// (decode_attn.cu: CUDA-core kernel; decode_mma.cu: tensor-core kernel for bf16 caches).
//
// A launch covers (sequence, kv-head, chunk of `chunk` positions) work units.  Each CTA builds
// the schedule itself (a warp scan over the sequences' lengths), walks units with a grid
// stride, and at the end of a unit merges its consumer warps' online-softmax states.  A unit
// that covers a whole sequence writes ctx; otherwise it writes its (o, m, l) partial and the
// last CTA to finish a (sequence, kv-head) merges all chunks of it (threadfence + arrival
// counter; nothing waits on anything).
#pragma once

#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace tl {

// chunks per sequence in one launch: the planners stay within it (64), and the merge
// weights of a sequence's chunks take kMaxChunksPerSeq * G floats of shared memory
constexpr int kMaxChunksPerSeq = 64;

__device__ __forceinline__ float safe_exp2_diff(float m, float M) {
    return (m == -INFINITY) ? 0.f : exp2f(m - M);
}

__device__ __forceinline__ size_t decode_partial_floats_dev(int total_units, int group, int d) {
    return (size_t)total_units * group * (d + 2);
}

struct Unit {
    int b, g, c, nch, n, p0, p1;
};

__device__ __forceinline__ int local_len(const DecodeArgs &a, int b, unsigned *err) {
    const int pos = a.pos[b];
    const int slice = a.kv.maxLen;
    if (pos < 0 || pos - a.pos_offset >= slice) {
        // single-GPU: the appended token must sit inside the cache (a split-KV shard only
        // covers part of the positions)
        if ((a.lse_out == nullptr && a.px.nranks == 0) || pos < 0) atomicOr(err, TL_DEVERR_POS_RANGE);
    }
    int n = pos + 1 - a.pos_offset;
    n = n < 0 ? 0 : (n > slice ? slice : n);
    return n;
}

__device__ __forceinline__ int nchunks(int n, int C) { return n <= 0 ? 1 : (n + C - 1) / C; }

__device__ __forceinline__ Unit decode_unit(const DecodeArgs &a, const int *prefix, const int *lens,
                                            int u) {
    Unit r;
    r.g = u % a.nHeadKv;
    const int t = u / a.nHeadKv;
    // upper_bound over prefix[0..nseq] for t
    int lo = 0, hi = a.nseq;  // prefix[lo] <= t < prefix[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] <= t) lo = mid; else hi = mid;
    }
    r.b = lo;
    r.c = t - prefix[lo];
    r.nch = prefix[lo + 1] - prefix[lo];
    r.n = lens[lo];
    r.p0 = r.c * a.chunk;
    r.p1 = min(r.p0 + a.chunk, r.n);
    if (r.p1 < r.p0) r.p1 = r.p0;
    return r;
}

// ---- dynamic unit schedule ---------------------------------------------------------------
// The producer warp of each CTA claims units from a.work[0] and hands their ids to the
// consumer warps through a small queue in shared memory (full/empty mbarriers), so a CTA that
// drew short units takes more of them.  Claims follow a rank order that puts every sequence's
// chunks before its last one first and the sequences' last chunks (the only partial ones)
// after them, so the units left for the final claims are the short ones.  The producer that
// finishes last resets the counters for the next launch.
constexpr int kUnitQ = 4;
struct UnitQueue {
    uint64_t full[kUnitQ], empty[kUnitQ];
    int id[kUnitQ];
};
constexpr int kUnitQBytes = (int)((sizeof(UnitQueue) + 15) / 16 * 16);

// Canonical unit index ((prefix[b] + c) * nHeadKv + g) of claim rank k.
__device__ __forceinline__ int unit_of_rank(const DecodeArgs &a, const int *prefix, int k) {
    const int H = a.nHeadKv;
    const int lead = (prefix[a.nseq] - a.nseq) * H;  // units of chunks other than a sequence's last
    if (k < lead) {
        const int t = k / H, g = k - t * H;
        // sequence b with prefix[b] - b <= t < prefix[b+1] - (b+1): the largest b with prefix[b] - b <= t
        int lo = 0, hi = a.nseq;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (prefix[mid] - mid <= t) lo = mid; else hi = mid;
        }
        return (prefix[lo] + (t - (prefix[lo] - lo))) * H + g;
    }
    const int r = k - lead;
    const int b = r / H, g = r - b * H;
    return (prefix[b + 1] - 1) * H + g;  // last chunk of sequence b
}

// Producer (one thread): claim the next unit and publish it; -1 when none remain.  Returns
// false if the wait for a free queue slot gave up (abort or timeout).
__device__ __forceinline__ bool unitq_push(const DecodeArgs &a, UnitQueue *q, const int *prefix, int total_units,
                                           int &slot, uint32_t &phase, int &u, bool &first, unsigned *err,
                                           volatile int *abort_flag) {
    // a CTA's first unit is its own rank (no round trip before the first copies); later ones
    // come from the counter, past the ranks the grid took that way
    const int k = first ? (int)blockIdx.x : (int)(gridDim.x + atomicAdd(a.work, 1u));
    first = false;
    u = k < total_units ? unit_of_rank(a, prefix, k) : -1;
    if (!mbar_wait(&q->empty[slot], phase ^ 1u, err, abort_flag)) return false;
    q->id[slot] = u;
    mbar_arrive(&q->full[slot]);
    if (++slot == kUnitQ) { slot = 0; phase ^= 1u; }
    return true;
}
// Producer, after publishing its -1: the last producer of the launch resets the counters.
__device__ __forceinline__ void unitq_finish(const DecodeArgs &a) {
    __threadfence();
    if (atomicAdd(a.work + 1, 1u) == gridDim.x - 1) {
        atomicExch(a.work, 0u);
        atomicExch(a.work + 1, 0u);
    }
}
// Consumer warp: the next unit id (the same for every lane), -1 at the end or on abort.
__device__ __forceinline__ int unitq_pop(UnitQueue *q, int &slot, uint32_t &phase, unsigned *err,
                                         volatile int *abort_flag, int lane) {
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&q->full[slot], phase, err, abort_flag));
    const int u = ok ? *reinterpret_cast<volatile int *>(&q->id[slot]) : -1;
    __syncwarp();
    if (lane == 0) mbar_arrive(&q->empty[slot]);
    if (++slot == kUnitQ) { slot = 0; phase ^= 1u; }
    return u;
}

// Warp 0: per-sequence local lengths, chunk counts and their exclusive prefix.
__device__ __forceinline__ void build_schedule(const DecodeArgs &a, int *prefix, int *lens, int *max_nch,
                                               int lane, unsigned *err) {
        const int per = (a.nseq + 31) / 32;
        const int s0 = lane * per, s1 = min(s0 + per, a.nseq);
        int sum = 0, mx = 0;
        for (int s = s0; s < s1; ++s) {
            const int n = local_len(a, s, err);
            lens[s] = n;
            sum += nchunks(n, a.chunk);
            mx = max(mx, nchunks(n, a.chunk));
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) max_nch[0] = mx;
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int run = incl - sum;
        for (int s = s0; s < s1; ++s) {
            prefix[s] = run;
            run += nchunks(lens[s], a.chunk);
        }
        if (lane == 31) prefix[a.nseq] = incl;
    }

// ---- split-KV across GPUs over peer memory ------------------------------------------------
// Exchange words: the float's bits in the low half, the call's epoch in the high half.
__device__ __forceinline__ void st_word_sys(unsigned long long *p, float v, unsigned epoch) {
    const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word_sys(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Has the word reached this call's epoch?  Epochs only grow.
__device__ __forceinline__ bool word_ready(unsigned long long w, unsigned epoch) {
    return (int)((unsigned)(w >> 32) - epoch) >= 0;
}
// Re-read a word until it carries this call's epoch, bounded by wait_ns from t0.  Returns the
// value, or 0 with *ok cleared (and the timeout bit set) on time-out.  Between reads the thread
// backs off: every consumer thread of the grid may be waiting here while other CTAs of this
// rank are still streaming their K/V, and a tight loop of system-scope loads would compete
// with that stream and with the peers' incoming stores.
__device__ __forceinline__ float wait_word(const unsigned long long *p, unsigned long long w, unsigned epoch,
                                           uint64_t t0, unsigned long long wait_ns, bool *ok, unsigned *err) {
    while (!word_ready(w, epoch)) {
        if (!*ok) return 0.f;
        if (globaltimer_ns() - t0 > wait_ns) {
            atomicOr(err, TL_DEVERR_TIMEOUT);
            *ok = false;
            return 0.f;
        }
        __nanosleep(128);
        w = ld_word_sys(p);
    }
    return __uint_as_float((unsigned)w);
}

// The final (o, m, l) of (sequence b, head) into slot `rank` of every rank's gather buffer
// (peer stores over NVLink; the own rank's entry is local memory).
template <int D>
__device__ __forceinline__ void peer_store_final(const DecodeArgs &a, int b, int head, int dd, float O, float M,
                                                 float L) {
    const int64_t row = (int64_t)a.px.rank * a.nseq * a.nHead + (int64_t)b * a.nHead + head;
    for (int r = 0; r < a.px.nranks; ++r) {
        unsigned long long *dst = a.px.gather[r] + row * (D + 2);
        st_word_sys(dst + dd, O, a.px.epoch);
        if (dd == 0) {
            st_word_sys(dst + D, M, a.px.epoch);
            st_word_sys(dst + D + 1, L, a.px.epoch);
        }
    }
}

// Four consecutive columns dd..dd+3 of the final (o, m, l) of (sequence b, head) into slot
// `rank` of rank r's gather buffer: two 16-byte vector stores of epoch-tagged words (each
// aligned 8-byte element of a vector store is written single-copy atomically, which is all
// the reader relies on), and m and l with column 0.
template <int D>
__device__ __forceinline__ void peer_store_group(const DecodeArgs &a, int r, int b, int head, int dd, float4 O,
                                                 float M, float L) {
    const int64_t row = (int64_t)a.px.rank * a.nseq * a.nHead + (int64_t)b * a.nHead + head;
    unsigned long long *dst = a.px.gather[r] + row * (D + 2) + dd;
    const unsigned long long ep = (unsigned long long)a.px.epoch << 32;
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(ep | __float_as_uint(O.x)),
                 "l"(ep | __float_as_uint(O.y))
                 : "memory");
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst + 2), "l"(ep | __float_as_uint(O.z)),
                 "l"(ep | __float_as_uint(O.w))
                 : "memory");
    if (dd == 0) {
        asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst + D), "l"(ep | __float_as_uint(M)),
                     "l"(ep | __float_as_uint(L))
                     : "memory");
    }
}

// After its own units, every consumer thread of the grid merges a share of this call's
// (sequence, head, column) elements, reading the ranks' words as they arrive:
//   M = max_r m_r,  L = sum_r l_r 2^(m_r - M),  ctx = sum_r o_r 2^(m_r - M) / L.
// The 3R words of an element are loaded together (one round trip), and only the ones that do
// not yet carry the call's epoch are read again.  A CTA waits only once its own units are
// done, and no rank's units wait on anything, so the waits cannot form a cycle.  Called by
// the NW*32 consumer threads.
template <int G, int D, int NW>
__device__ __forceinline__ void peer_merge_pairs(const DecodeArgs &a, int tid) {
    const int R = a.px.nranks;
    const unsigned long long *g = a.px.gather[a.px.rank];
    const int64_t stride = (int64_t)a.nseq * a.nHead * (D + 2);
    const int64_t total = (int64_t)a.nseq * a.nHead * D;
    const unsigned epoch = a.px.epoch;
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    for (int64_t e = (int64_t)blockIdx.x * (NW * 32) + tid; e < total && ok; e += (int64_t)gridDim.x * (NW * 32)) {
        const int64_t row = e / D;
        const int dd = (int)(e - row * D);
        const unsigned long long *pr = g + row * (D + 2);
        unsigned long long wm[kMaxPeers], wl[kMaxPeers], wo[kMaxPeers];
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r) {
            if (r < R) {
                wm[r] = ld_word_sys(pr + r * stride + D);
                wl[r] = ld_word_sys(pr + r * stride + D + 1);
                wo[r] = ld_word_sys(pr + r * stride + dd);
            }
        }
        float m[kMaxPeers], l[kMaxPeers], o[kMaxPeers];
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r) {
            if (r >= R) break;
            m[r] = wait_word(pr + r * stride + D, wm[r], epoch, t0, a.px.wait_ns, &ok, a.err);
            l[r] = wait_word(pr + r * stride + D + 1, wl[r], epoch, t0, a.px.wait_ns, &ok, a.err);
            o[r] = wait_word(pr + r * stride + dd, wo[r], epoch, t0, a.px.wait_ns, &ok, a.err);
            M = fmaxf(M, m[r]);
        }
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r) {
            if (r >= R) break;
            const float w = safe_exp2_diff(m[r], M);
            L = fmaf(l[r], w, L);
            O = fmaf(o[r], w, O);
        }
        if (ok) a.out[row * D + dd] = (L > 0.f) ? O / L : 0.f;
    }
}

// Merge of the NW consumer warps' states (written to wm[NW][G], wl[NW][G], wo[NW][G][D]) at the
// end of unit u, then the cross-chunk merge by the last CTA.  Called by the NW*32 consumer
// threads of the CTA; uses named barrier 1.
template <int G, int D, int NW>
__device__ __forceinline__ void unit_epilogue(const DecodeArgs &a, const Unit &un, int u, const int *prefix,
                                              float *wm, float *wl, float *wo, float *cw, int *is_last_flag,
                                              int tid, int warp, int lane) {
        named_bar(1, NW * 32);
        const bool peer = a.px.nranks > 0;
        const bool single = (un.nch == 1) && (a.lse_out == nullptr) && !peer;
        const int unit_index = u;  // partial slot of this unit
        for (int e = tid; e < G * D; e += NW * 32) {
            const int h = e / D, dd = e - h * D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w * G + h]);
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float sw = safe_exp2_diff(wm[w * G + h], M);
                L = fmaf(wl[w * G + h], sw, L);
                O = fmaf(wo[(w * G + h) * D + dd], sw, O);
            }
            const int head = un.g * G + h;
            if (single) {
                a.out[((int64_t)un.b * a.nHead + head) * D + dd] = (L > 0.f) ? O / L : 0.f;
            } else if (un.nch == 1 && peer) {
                peer_store_final<D>(a, un.b, head, dd, O, M, L);
            } else if (un.nch == 1) {
                float *dst = a.lse_out + ((int64_t)un.b * a.nHead + head) * (D + 2);
                dst[dd] = O;
                if (dd == 0) { dst[D] = M; dst[D + 1] = L; }
            } else {
                float *dst = a.partial + ((int64_t)unit_index * G + h) * (D + 2);
                dst[dd] = O;
                if (dd == 0) { dst[D] = M; dst[D + 1] = L; }
            }
        }
        if (un.nch > 1) {
            __threadfence();
            named_bar(1, NW * 32);
            if (tid == 0) {
                const unsigned old = atomicAdd(&a.counter[un.b * a.nHeadKv + un.g], 1u);
                *is_last_flag = (old == (unsigned)(un.nch - 1)) ? 1 : 0;
            }
            named_bar(1, NW * 32);
            if (*is_last_flag) {
                __threadfence();
                // per-head max / sum over the chunks (warp h handles heads h, h+4, ...)
                for (int h = warp; h < G; h += NW) {
                    float M = -INFINITY;
                    for (int c = lane; c < un.nch; c += 32) {
                        const int uc = (prefix[un.b] + c) * a.nHeadKv + un.g;
                        M = fmaxf(M, __ldcg(&a.partial[((int64_t)uc * G + h) * (D + 2) + D]));
                    }
#pragma unroll
                    for (int o2 = 16; o2 >= 1; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
                    float L = 0.f;
                    for (int c = lane; c < un.nch; c += 32) {
                        const int uc = (prefix[un.b] + c) * a.nHeadKv + un.g;
                        const float *pp = &a.partial[((int64_t)uc * G + h) * (D + 2) + D];
                        const float w = safe_exp2_diff(__ldcg(pp), M);
                        cw[c * G + h] = w;
                        L = fmaf(__ldcg(pp + 1), w, L);
                    }
#pragma unroll
                    for (int o2 = 16; o2 >= 1; o2 >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o2);
                    if (lane == 0) { wm[h] = M; wl[h] = L; }
                }
                named_bar(1, NW * 32);
                for (int e = tid; e < G * D; e += NW * 32) {
                    const int h = e / D, dd = e - h * D;
                    float O = 0.f;
                    // partials of consecutive chunks are a fixed stride apart; four independent
                    // accumulators keep several L2 loads in flight
                    const int64_t stride = (int64_t)a.nHeadKv * G * (D + 2);
                    const float *src = a.partial + ((int64_t)(prefix[un.b] * a.nHeadKv + un.g) * G + h) * (D + 2) + dd;
                    float O1 = 0.f, O2 = 0.f, O3 = 0.f;
                    int c = 0;
                    for (; c + 4 <= un.nch; c += 4) {
                        const float x0 = __ldcg(src + (c + 0) * stride), x1 = __ldcg(src + (c + 1) * stride);
                        const float x2 = __ldcg(src + (c + 2) * stride), x3 = __ldcg(src + (c + 3) * stride);
                        O = fmaf(cw[(c + 0) * G + h], x0, O);
                        O1 = fmaf(cw[(c + 1) * G + h], x1, O1);
                        O2 = fmaf(cw[(c + 2) * G + h], x2, O2);
                        O3 = fmaf(cw[(c + 3) * G + h], x3, O3);
                    }
                    for (; c < un.nch; ++c) O = fmaf(cw[c * G + h], __ldcg(src + c * stride), O);
                    O = (O + O1) + (O2 + O3);
                    const int head = un.g * G + h;
                    const float L = wl[h];
                    if (peer) {
                        peer_store_final<D>(a, un.b, head, dd, O, wm[h], L);
                    } else if (a.lse_out == nullptr) {
                        a.out[((int64_t)un.b * a.nHead + head) * D + dd] = (L > 0.f) ? O / L : 0.f;
                    } else {
                        float *dst = a.lse_out + ((int64_t)un.b * a.nHead + head) * (D + 2);
                        dst[dd] = O;
                        if (dd == 0) { dst[D] = wm[h]; dst[D + 1] = L; }
                    }
                }
                if (tid == 0) a.counter[un.b * a.nHeadKv + un.g] = 0u;
            }
        }
}

}  // namespace tl
