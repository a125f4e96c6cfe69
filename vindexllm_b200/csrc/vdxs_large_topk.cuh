// vdxs_large_topk.cuh - the top-k path for 1024 < top_k < V (Sampler.pas:327-459 with a
// K-slot buffer larger than the shared-memory paths hold). Included by vdxs_kernels.cu
// inside namespace vdxs, after the block primitives, block_select, block_emit, the
// stage-1 list source (ListSrc) and the stream kernel's constants.
//
// One 256-thread CTA per row (a persistent grid walks the rows), with a per-CTA
// workspace in global memory of 24 bytes per slot:
//   1. the row maximum, then an exact radix select of the K best (key desc, index asc)
//      elements and their compaction, over the row's stage-1 list and penalised entries
//      when the stream kernel ran first (32 K <= V) and the list is complete, else over
//      the row in global memory (penalised values overlaid from the per-row bitmap and
//      the sorted penalty lists);
//   2. probabilities, min-p, a single-CTA LSD radix sort of (probability, ~index) keys,
//      and the reference's sequential double walk (Sampler.pas:385-459) by one thread
//      over values staged through shared memory: the canonical token;
//   3. in faithful mode, rows whose reference token can depend on the K-slot buffer's
//      slot history re-run the min-buffer (Sampler.pas:341-383) with a 32-ary
//      tournament tree over the slots, then the reference tail in slot order.

constexpr int kLkItems = 4;                       // keys per thread per radix-sort tile
constexpr int kLkTile = kLkItems * NT;            // keys per radix-sort tile
constexpr int kLkTab = kLkItems * NWARPS * 256;   // per-(item, warp, digit) counts of a tile
constexpr int kLkStage = 2048;                    // values per staged chunk of a sequential walk
constexpr int kLkSmemTreeMax = 8192 + 256 + 8 + 1;  // tree nodes kept in shared memory (K <= 2^18)
static_assert(NT == 256, "the radix sort gives one thread per digit value");

// Tree levels above the slots: level sizes ceil(K/32), ceil(K/1024), ... down to 1.
__host__ __device__ inline int lk_tree_nodes(int K) {
    int total = 0;
    for (int n = (K + 31) / 32;; n = (n + 31) / 32) {
        total += n;
        if (n == 1) break;
    }
    return total;
}

__host__ __device__ inline size_t lk_smem_bytes(int K) {
    const size_t tree = lk_tree_nodes(K) <= kLkSmemTreeMax ? (size_t)8 * lk_tree_nodes(K) : 0;
    const size_t uni = std::max((size_t)4 * kLkTab, tree);
    return kHeadBytes + (size_t)4 * 8 * 256 + (size_t)4 * 256 + (size_t)4 * kLkStage + uni;
}

// 64-bit words of one CTA's global workspace: two sort buffers of K keys, K (key, index)
// slots, and the tree levels when they do not fit in shared memory.
__host__ __device__ inline int64_t lk_cta_words(int K) {
    const int64_t tree = lk_tree_nodes(K) <= kLkSmemTreeMax ? 0 : lk_tree_nodes(K);
    return 3 * (int64_t)K + tree;
}

// A row in global memory with the penalised values overlaid (bitmap of the penalised
// local ids, then a binary search in the sorted unique id list). NaN: no element.
template <typename T>
struct PenRowSrc {
    const T* row;
    const uint32_t* bits;  // null when no penalty applies
    const int32_t* pid;
    const float* pvl;
    int npen;
    __device__ __forceinline__ float val(int i) const {
        if (bits && ((bits[i >> 5] >> (i & 31)) & 1u)) return pvl[lower_bound_i32(pid, npen, i)];
        return ld_elem(row, i);
    }
    __device__ __forceinline__ uint32_t key(int i) const {
        const float v = val(i);
        return v == v ? f2key(v) : 0u;
    }
    __device__ __forceinline__ uint32_t tb(int i) const { return (uint32_t)i; }
};

// Stable LSD radix sort of n 64-bit keys into descending order, by the whole CTA.
// a and b are global buffers of n keys; the result is in the returned one. dh: 8 x 256
// digit counts, base: 256 bucket offsets, tab: kLkTab counts, sh: block scratch.
__device__ uint64_t* lk_sort_desc(uint64_t* a, uint64_t* b, int n, uint32_t* dh, uint32_t* base, uint32_t* tab,
                                  int* sh) {
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int i = tid; i < 8 * 256; i += NT) dh[i] = 0u;
    __syncthreads();
    // All eight digit histograms in one pass (ascending order of ~key is descending order
    // of key); equal digits of a warp are counted with one atomic.
    for (int i0 = 0; i0 < n; i0 += NT) {
        const int i = i0 + tid;
        const uint64_t k = i < n ? ~a[i] : 0ull;
#pragma unroll
        for (int d = 0; d < 8; ++d) {
            const int dg = i < n ? (int)((k >> (8 * d)) & 255u) : 256;
            const unsigned peers = __match_any_sync(FULL, dg);
            if (dg < 256 && (peers & lanemask_lt()) == 0u) atomicAdd(&dh[d * 256 + dg], (uint32_t)__popc(peers));
        }
    }
    __syncthreads();
    uint64_t* src = a;
    uint64_t* dst = b;
    for (int d = 0; d < 8; ++d) {
        const uint32_t c = dh[d * 256 + tid];
        if (__syncthreads_or(c == (uint32_t)n)) continue;  // every key has this digit
        int tot;
        base[tid] = (uint32_t)block_excl_scan((int)c, sh, &tot);
        const int shift = 8 * d;
        for (int t0 = 0; t0 < n; t0 += kLkTile) {
            for (int i = tid; i < kLkTab; i += NT) tab[i] = 0u;
            __syncthreads();
            uint64_t kk[kLkItems];
            int dg[kLkItems], rk[kLkItems];
#pragma unroll
            for (int u = 0; u < kLkItems; ++u) {
                const int i = t0 + u * NT + tid;
                kk[u] = i < n ? src[i] : 0ull;
                dg[u] = i < n ? (int)((~kk[u] >> shift) & 255u) : 256;
                const unsigned peers = __match_any_sync(FULL, dg[u]);
                rk[u] = __popc(peers & lanemask_lt());
                if (dg[u] < 256 && rk[u] == 0) tab[(u * NWARPS + warp) * 256 + dg[u]] = (uint32_t)__popc(peers);
            }
            __syncthreads();
            // Thread t owns digit t: offsets in position order (item, warp), then the
            // bucket's running base for the next tile.
            uint32_t run = base[tid];
            for (int j = 0; j < kLkItems * NWARPS; ++j) {
                const uint32_t x = tab[j * 256 + tid];
                tab[j * 256 + tid] = run;
                run += x;
            }
            base[tid] = run;
            __syncthreads();
#pragma unroll
            for (int u = 0; u < kLkItems; ++u)
                if (dg[u] < 256) dst[tab[(u * NWARPS + warp) * 256 + dg[u]] + rk[u]] = kk[u];
            __syncthreads();
        }
        uint64_t* t = src;
        src = dst;
        dst = t;
    }
    __syncthreads();
    return src;
}

// Thread 0 visits f(i, v) for i = 0, 1, ..., n-1 in order and stops when f returns false;
// the values come from get(i), staged through shared memory by the whole CTA.
template <class G, class F>
__device__ void lk_walk(int n, float* stage, int* stop, G get, F f) {
    if (threadIdx.x == 0) *stop = 0;
    __syncthreads();
    for (int c0 = 0; c0 < n; c0 += kLkStage) {
        const int m = min(kLkStage, n - c0);
        for (int i = threadIdx.x; i < m; i += NT) stage[i] = get(c0 + i);
        __syncthreads();
        if (threadIdx.x == 0)
            for (int i = 0; i < m; ++i)
                if (!f(c0 + i, stage[i])) {
                    *stop = 1;
                    break;
                }
        __syncthreads();
        if (*stop) break;
    }
    __syncthreads();
}

__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
    const uint32_t hi = __reduce_min_sync(FULL, (uint32_t)(v >> 32));
    const uint32_t lo = __reduce_min_sync(FULL, (uint32_t)(v >> 32) == hi ? (uint32_t)v : 0xFFFFFFFFu);
    return ((uint64_t)hi << 32) | lo;
}

// Walk of n walk-ordered probabilities (Sampler.pas:412-459): sequential double sums, the
// top-p cut when `sorted`, and the draw. Thread 0's results are published in r[].
struct LkWalk {
    int j;            // drawn walk position, -1 = no crossing (fallback)
    int m;            // walk positions kept by top-p
    double t, lsum, before, total, c_prev, c_m;
    float q_m;        // probability at position m (0 when m == n)
};

template <class G>
__device__ void lk_draw_walk(int n, bool sorted, float top_p, float u, float* stage, int* stop, G get, LkWalk* r) {
    double total = 0.0;
    lk_walk(n, stage, stop, get, [&](int, float v) {
        total += v;
        return true;
    });
    int m = n;
    double lsum = total, c_prev = 0.0, c_m = total;
    float q_m = 0.0f;
    if (sorted) {
        const double target = (double)top_p * total;
        double cum = 0.0;
        lsum = 0.0;
        m = 0;
        lk_walk(n, stage, stop, get, [&](int i, float v) {
            if (cum < target && v > 0.0f) {
                c_prev = cum;
                cum += v;
                lsum += v;
                m = i + 1;
                return true;
            }
            q_m = v;
            return false;
        });
        c_m = cum;
        // Only thread 0 walked: every thread takes its cut for the draw's (uniform) bound.
        if (threadIdx.x == 0) r->m = m;
        __syncthreads();
        m = r->m;
    }
    const double t = (double)u * lsum;
    double cum = 0.0, before = 0.0;
    int j = -1;
    lk_walk(m, stage, stop, get, [&](int i, float v) {
        before = cum;
        cum += v;
        if (cum > t) {
            j = i;
            return false;
        }
        return true;
    });
    if (threadIdx.x == 0) {
        r->j = j;
        r->m = m;
        r->t = t;
        r->lsum = lsum;
        r->before = before;
        r->total = total;
        r->c_prev = c_prev;
        r->c_m = c_m;
        r->q_m = q_m;
    }
    __syncthreads();
}

// The min-buffer emulation and the reference tail for one row (faithful mode).
template <typename T>
__device__ void lk_faithful_row(const KParams& p, int b, const PenRowSrc<T>& src, uint32_t kmax, uint32_t flags_in,
                                uint64_t* sa, uint64_t* sb, uint32_t* sk, int32_t* si, uint64_t* tree,
                                unsigned char* smem_base, uint32_t* dh, uint32_t* base, uint32_t* tab, float* stage,
                                uint32_t* shu, int* sh_i) {
    const int tid = threadIdx.x, lane = tid & 31;
    const int K = p.K, V = p.V;
    (void)smem_base;
    // Level sizes and offsets of the tree over the slots (level 0 = the slots themselves).
    int nl = 0, lsz[8], loff[8];
    {
        int off = 0;
        for (int n = (K + 31) / 32;; n = (n + 31) / 32) {
            lsz[nl] = n;
            loff[nl] = off;
            off += n;
            ++nl;
            if (n == 1) break;
        }
    }
    // The first K elements fill the slots in order (Sampler.pas:352-356).
    for (int s = tid; s < K; s += NT) {
        sk[s] = src.key(s);
        si[s] = s;
    }
    __syncthreads();
    auto slot_comp = [&](int s) -> uint64_t { return ((uint64_t)sk[s] << 32) | (uint32_t)s; };
    for (int l = 0; l < nl; ++l) {
        const int nchild = l == 0 ? K : lsz[l - 1];
        for (int g = tid; g < lsz[l]; g += NT) {
            uint64_t mn = ~0ull;
            for (int c = 32 * g; c < min(32 * g + 32, nchild); ++c)
                mn = min(mn, l == 0 ? slot_comp(c) : tree[loff[l - 1] + c]);
            tree[loff[l] + g] = mn;
        }
        __syncthreads();
    }
    // The rest of the row in index order (Sampler.pas:358-383): an element strictly above
    // the minimum replaces the minimum's slot; the minimum is the smallest key, lowest
    // slot first (the reference's first slot with a strict '<').
    if (tid < 32) {
        uint64_t mn = tree[loff[nl - 1]];
        constexpr int U = 4;
        for (int64_t i0 = K; i0 < V; i0 += 32 * U) {
            uint32_t kk[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t i = i0 + u * 32 + lane;
                kk[u] = i < V ? src.key((int)i) : 0u;
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                unsigned pend = __ballot_sync(FULL, kk[u] > (uint32_t)(mn >> 32));
                while (pend) {
                    const int l = __ffs(pend) - 1;
                    const uint32_t nk = __shfl_sync(FULL, kk[u], l);
                    const int s = (int)(uint32_t)mn;
                    if (lane == 0) {
                        sk[s] = nk;
                        si[s] = (int32_t)(i0 + u * 32 + l);
                    }
                    // Path to the root: each level's node is the minimum of its 32 children.
                    uint64_t c = ((uint64_t)nk << 32) | (uint32_t)s;
                    int g = s;
                    for (int lv = 0; lv < nl; ++lv) {
                        const int parent = g >> 5, child = 32 * parent + lane;
                        const int nchild = lv == 0 ? K : lsz[lv - 1];
                        uint64_t x = ~0ull;
                        if (child == g) x = c;
                        else if (child < nchild) x = lv == 0 ? slot_comp(child) : tree[loff[lv - 1] + child];
                        c = warp_min_u64(x);
                        if (lane == 0) tree[loff[lv] + parent] = c;
                        __syncwarp();
                        g = parent;
                    }
                    mn = c;
                    pend &= ~(1u << l);
                    pend &= __ballot_sync(FULL, kk[u] > (uint32_t)(mn >> 32));
                }
            }
        }
    }
    __syncthreads();

    // Reference tail in slot order (Sampler.pas:385-459). The maximum over all elements
    // is in the buffer, so kmax is the buffer's largest key.
    const double Md = (double)key2f(kmax), it = (double)p.inv_temp;
    float* prob = (float*)sk;  // probabilities replace the slot keys
    for (int s = tid; s < K; s += NT) prob[s] = (float)exp(((double)key2f(sk[s]) - Md) * it);
    __syncthreads();
    if (p.min_p > 0.0f) {
        uint32_t mk = 0u;
        for (int s = tid; s < K; s += NT) mk = max(mk, f2key(prob[s]));
        mk = block_max_u32(mk, shu);
        const float thr = __fmul_rn(key2f(mk), p.min_p);
        for (int s = tid; s < K; s += NT)
            if (prob[s] < thr) prob[s] = 0.0f;
        __syncthreads();
    }
    const bool sorted = p.top_p < 1.0f;
    const uint64_t* wo = nullptr;  // walk order when sorted: (probability, 0xFFFFFFFF - slot)
    if (sorted) {
        // Stable descending insertion sort == sort by (prob desc, slot asc).
        for (int s = tid; s < K; s += NT)
            sa[s] = ((uint64_t)__float_as_uint(prob[s]) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)s);
        __syncthreads();
        wo = lk_sort_desc(sa, sb, K, dh, base, tab, sh_i);
    }
    auto wprob = [&](int i) -> float { return sorted ? __uint_as_float((uint32_t)(wo[i] >> 32)) : prob[i]; };
    auto wid = [&](int i) -> int32_t { return sorted ? si[0xFFFFFFFFu - (uint32_t)wo[i]] : si[i]; };
    for (int s = tid; s < p.out_k; s += NT) {
        if (p.out_idx) p.out_idx[(int64_t)b * p.out_k + s] = s < K ? wid(s) : -1;
        if (p.out_prob) p.out_prob[(int64_t)b * p.out_k + s] = s < K ? wprob(s) : 0.0f;
    }
    // The slot-order sum also covers min-p: zeroed entries add nothing to a double sum.
    __shared__ LkWalk s_w;
    const float u = p.uniform ? p.uniform[b] : 0.0f;
    lk_draw_walk(K, sorted, p.top_p, u, stage, sh_i + 16, wprob, &s_w);
    if (tid == 0) {
        int j = s_w.j;
        const bool fallback = j < 0;
        if (fallback) j = K - 1;
        uint32_t f = (flags_in & (VDXS_FLAG_BOUNDARY_TIE | VDXS_FLAG_INEXACT_SUM)) | VDXS_FLAG_TOPK |
                     VDXS_FLAG_FAITHFUL_PASS;
        if (!sorted) f |= VDXS_FLAG_SLOT_ORDER;
        if (fallback) f |= VDXS_FLAG_FALLBACK;
        if (sorted && ((j > 0 && wprob(j - 1) == wprob(j)) || (j + 1 < K && wprob(j + 1) == wprob(j))))
            f |= VDXS_FLAG_DRAW_TIE_RUN;
        const double before = s_w.before, t = s_w.t, lsum = s_w.lsum;
        const double after = before + (fallback ? 0.0 : (double)wprob(j));
        const double eps = 1e-6 * lsum;
        if (fallback || (t - before) <= eps || (after - t) <= eps) f |= VDXS_FLAG_NEAR_BOUNDARY;
        p.tokens[b] = wid(j);
        if (p.flags) p.flags[b] = f;
    }
    __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(NT) topk_large_kernel(KParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t* hist = (uint32_t*)smem_raw;
    uint32_t* sh = hist + kHistWords;
    uint32_t* dh = (uint32_t*)(smem_raw + kHeadBytes);
    uint32_t* base = dh + 8 * 256;
    float* stage = (float*)(base + 256);
    unsigned char* uni = (unsigned char*)(stage + kLkStage);
    uint32_t* tab = (uint32_t*)uni;
    const int tid = threadIdx.x;
    const int K = p.K, V = p.V;
    const int64_t words = lk_cta_words(K);
    uint64_t* ws = p.lk_buf + (int64_t)blockIdx.x * words;
    uint64_t* sa = ws;
    uint64_t* sb = ws + K;
    uint32_t* ck = (uint32_t*)(ws + 2 * (int64_t)K);
    uint32_t* ci = ck + K;
    uint64_t* tree = lk_tree_nodes(K) <= kLkSmemTreeMax ? (uint64_t*)uni : ws + 3 * (int64_t)K;
    int* sh_i = (int*)(sh + 40);  // block_excl_scan scratch (NWARPS ints) and the walk's stop flag
    const int tbb = bits_for((uint32_t)(V - 1));
    for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
        const int npen = p.pen_cnt ? p.pen_cnt[b] : 0;
        const PenRowSrc<T> src{(const T*)p.logits + (int64_t)b * p.stride,
                               p.pen_bits && npen > 0 ? p.pen_bits + (int64_t)b * p.pen_words : nullptr,
                               p.pen_ids ? p.pen_ids + (int64_t)b * p.pen_stride : nullptr,
                               p.pen_vals ? p.pen_vals + (int64_t)b * p.pen_stride : nullptr, npen};
        // 1. Row maximum and the exact top K in (key desc, index asc) order, from the row's
        //    stage-1 list when stage 1 ran and the list is complete, else from the row.
        auto top_k = [&](const auto& sel, int n, auto idx_of, int tbits, uint32_t* kmax_out) -> SelectOut {
            uint32_t km = 0u;
            for (int i0 = tid; i0 < n; i0 += 4 * NT) {
                uint32_t k[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) k[u] = i0 + u * NT < n ? sel.key(i0 + u * NT) : 0u;
                km = max(max(km, max(k[0], k[1])), max(k[2], k[3]));
            }
            *kmax_out = block_max_u32(km, sh + 32);
            const SelectOut so = block_select(sel, n, K, *kmax_out, tbits, hist, sh);
            sh[60] = (uint32_t)block_emit(sel, n, so, ck, ci, K, &sh[8], idx_of);
            __syncthreads();
            return so;
        };
        uint32_t kmax;
        SelectOut s;
        const uint32_t lcount = p.lk_list ? __ldcg(&p.row_cnt[b]) : 0u;
        if (p.lk_list && lcount <= (uint32_t)p.cand_cap) {
            const ListSrc ls{p.cand + (int64_t)b * p.cand_cap, (int)lcount,
                             __ldcg(&p.row_tau[(int64_t)b * kTauStride]), src.pid, src.pvl, p.vocab_offset};
            s = top_k(ls, (int)lcount + npen, ListIdx{&ls}, bits_for((uint32_t)(p.vocab_offset + V - 1)), &kmax);
        } else {
            s = top_k(src, V, OffsetIdx{(uint32_t)p.vocab_offset}, tbb, &kmax);
        }
        const int nsel = (int)sh[60];
        __syncthreads();
        uint32_t kb = 0xFFFFFFFFu;
        for (int i = tid; i < nsel; i += NT) kb = min(kb, ck[i]);
        kb = block_min_u32(kb, sh + 32);
        const uint32_t btie = s.tie_cut ? VDXS_FLAG_BOUNDARY_TIE : 0u;
        if (nsel == 0) {
            // No element compares (every value NaN): the reference's fallback slot.
            if (tid == 0) {
                p.tokens[b] = K - 1;
                if (p.flags) p.flags[b] = VDXS_FLAG_TOPK | VDXS_FLAG_FALLBACK | VDXS_FLAG_NEAR_BOUNDARY;
            }
            for (int i = tid; i < p.out_k; i += NT) {
                if (p.out_idx) p.out_idx[(int64_t)b * p.out_k + i] = -1;
                if (p.out_prob) p.out_prob[(int64_t)b * p.out_k + i] = 0.0f;
            }
            __syncthreads();
            continue;
        }

        // 2. Probabilities (fp64 exp rounded to fp32), min-p, the walk order
        //    (probability desc, index asc), the reference's sequential arithmetic.
        const double Md = (double)key2f(kmax), it = (double)p.inv_temp;
        float* q = (float*)ck;
        for (int i = tid; i < nsel; i += NT) q[i] = (float)exp(((double)key2f(ck[i]) - Md) * it);
        float qb = kb != 0xFFFFFFFFu ? (float)exp(((double)key2f(kb) - Md) * it) : -1.0f;
        __syncthreads();
        if (p.min_p > 0.0f) {
            uint32_t mk = 0u;
            for (int i = tid; i < nsel; i += NT) mk = max(mk, f2key(q[i]));
            mk = block_max_u32(mk, sh + 32);
            const float thr = __fmul_rn(key2f(mk), p.min_p);
            for (int i = tid; i < nsel; i += NT)
                if (q[i] < thr) q[i] = 0.0f;
            if (qb >= 0.0f && qb < thr) qb = 0.0f;
            __syncthreads();
        }
        for (int i = tid; i < nsel; i += NT) sa[i] = ((uint64_t)__float_as_uint(q[i]) << 32) | (uint64_t)(~ci[i]);
        __syncthreads();
        const uint64_t* wo = lk_sort_desc(sa, sb, nsel, dh, base, tab, sh_i);
        auto wq = [&](int i) -> float { return __uint_as_float((uint32_t)(wo[i] >> 32)); };
        auto wid = [&](int i) -> int32_t { return (int32_t)~(uint32_t)wo[i]; };
        // Exactness of the double sums (any order gives the same result).
        uint32_t cnt = 0u, emin = 0xFFFFFFFFu;
        for (int i = tid; i < nsel; i += NT) {
            const float v = wq(i);
            if (v > 0.0f) {
                ++cnt;
                int e = ilogbf(v);
                e = e < -126 ? -126 : e;
                emin = min(emin, (uint32_t)(e + 1024));
            }
        }
        cnt = block_sum_u32(cnt, sh + 32);
        emin = block_min_u32(emin, sh + 32);
        bool exact = true;
        if (cnt > 0u) exact = (int)emin - 1024 >= ilogb((double)cnt * (double)wq(0)) - 29;
        __shared__ LkWalk s_w;
        const float uu = p.uniform ? p.uniform[b] : 0.0f;
        const bool sorted = p.top_p < 1.0f;
        lk_draw_walk(nsel, sorted, p.top_p, uu, stage, sh_i + 16, wq, &s_w);
        int j = s_w.j;
        const bool fallback = j < 0;
        if (fallback) j = nsel - 1;
        uint32_t f = btie | VDXS_FLAG_TOPK;
        if (!exact) f |= VDXS_FLAG_INEXACT_SUM;
        if (!sorted && K > 1) f |= VDXS_FLAG_SLOT_ORDER;
        if (fallback) f |= VDXS_FLAG_FALLBACK;
        const float qj = wq(j);
        if (nsel > 1 && ((j > 0 && wq(j - 1) == qj) || (j + 1 < nsel && wq(j + 1) == qj)))
            f |= VDXS_FLAG_DRAW_TIE_RUN;
        {
            const double after = s_w.before + (fallback ? 0.0 : (double)qj);
            const double eps = 1e-6 * s_w.lsum;
            if (fallback || (s_w.t - s_w.before) <= eps || (after - s_w.t) <= eps) f |= VDXS_FLAG_NEAR_BOUNDARY;
        }
        bool need_faithful = false;
        if (p.tie_mode == VDXS_TIES_FAITHFUL && K > 1) {
            const bool boundary_draw = btie && qj == qb;
            need_faithful = boundary_draw || (f & (VDXS_FLAG_DRAW_TIE_RUN | VDXS_FLAG_SLOT_ORDER));
            if (!need_faithful && !exact) {
                // The reference sums in slot order, this walk in probability order. Both
                // are recursive double sums of the same cnt terms, each within
                // (cnt - 1) * 2^-53 * total of the exact sum, and they only reach the
                // token through the top-p target. The token is the reference's when no
                // walk decision lies within that distance of the target; otherwise the
                // row is re-resolved.
                const double S = s_w.total, tc = (double)p.top_p * S;
                const double dS = 2.0 * ((double)cnt + 1.0) * 0x1p-53 * S * (1.0 + 0x1p-20);
                const double dt = (double)p.top_p * dS + 0x1p-51 * tc;
                const int m = s_w.m;
                const bool ok_prev = m == 0 || s_w.c_prev < tc - dt;
                const bool ok_stop = m == nsel || s_w.q_m == 0.0f || s_w.c_m >= tc + dt;
                need_faithful = !(ok_prev && ok_stop);
            }
        }
        if (!need_faithful) {
            if (tid == 0) {
                p.tokens[b] = wid(j);
                if (p.flags) p.flags[b] = f;
            }
            for (int i = tid; i < p.out_k; i += NT) {
                if (p.out_idx) p.out_idx[(int64_t)b * p.out_k + i] = i < nsel ? wid(i) : -1;
                if (p.out_prob) p.out_prob[(int64_t)b * p.out_k + i] = i < nsel ? wq(i) : 0.0f;
            }
        } else {
            lk_faithful_row<T>(p, b, src, kmax, f, sa, sb, ck, (int32_t*)ci, tree, smem_raw, dh, base, tab, stage,
                               sh + 32, sh_i);
        }
        __syncthreads();
        // The row's penalised-id bitmap words are left at zero for the next call, and after
        // a stage-1 pass its bound, list count and key histogram as well.
        if (src.bits)
            for (int jx = tid; jx < npen; jx += NT) p.pen_bits[(int64_t)b * p.pen_words + (src.pid[jx] >> 5)] = 0u;
        if (p.lk_list) {
            if (tid == 0) {
                p.row_tau[(int64_t)b * kTauStride] = 0u;
                p.row_cnt[b] = 0u;
            }
            uint4* rh4 = reinterpret_cast<uint4*>(p.rhist + (int64_t)b * kRowHistWords);
            for (int i = tid; i < kRowHistWords / 4; i += NT) rh4[i] = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncthreads();
    }
}
