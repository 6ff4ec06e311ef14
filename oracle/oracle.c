/*
 * CPU oracle for the InfLLM-v2 block-selection path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, the
 * smoke check and the CPU-baseline leg of bench.py compare against.  The
 * product path (unum_ops_b200) never links, loads or calls it.
 *
 * Each function restates one step of the reference (Yanguan619/unum_ops,
 * Python/Triton) in plain C, citing the reference lines it follows.  The
 * restatement is pinned against outputs of the reference itself, produced in
 * the build container by tests/golden/make_golden.py and committed as
 * fixtures under tests/golden/.
 *
 * Threading: the loops over independent rows run on a small pthread pool so
 * the same code serves as the timed CPU baseline; results do not depend on
 * the thread count (each output element is produced by exactly one thread,
 * with a fixed summation order).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>

static int g_threads = 1;

int oracle_num_threads(void) { return g_threads; }

void oracle_set_num_threads(int n) {
    if (n <= 0) {
        long c = sysconf(_SC_NPROCESSORS_ONLN);
        n = c > 0 ? (int)c : 1;
    }
    g_threads = n;
}

/* Parallel for over [0, n): workers take chunks of `chunk` rows from a shared
 * atomic counter.  fn(begin, end, ctx) handles one chunk. */
typedef void (*range_fn)(int64_t, int64_t, void *);
typedef struct {
    range_fn fn;
    void *ctx;
    int64_t n, chunk;
    atomic_llong next;
} pool_job;

static void *pool_worker(void *arg) {
    pool_job *job = (pool_job *)arg;
    for (;;) {
        int64_t b = atomic_fetch_add(&job->next, job->chunk);
        if (b >= job->n) break;
        int64_t e = b + job->chunk < job->n ? b + job->chunk : job->n;
        job->fn(b, e, job->ctx);
    }
    return NULL;
}

static void parallel_for(int64_t n, int64_t chunk, range_fn fn, void *ctx) {
    if (n <= 0) return;
    pool_job job;
    job.fn = fn;
    job.ctx = ctx;
    job.n = n;
    job.chunk = chunk > 0 ? chunk : 1;
    atomic_init(&job.next, 0);
    int nt = g_threads;
    if (nt <= 1 || n <= job.chunk) {
        pool_worker(&job);
        return;
    }
    pthread_t th[256];
    if (nt > 256) nt = 256;
    int started = 0;
    for (int i = 1; i < nt; ++i)
        if (pthread_create(&th[started], NULL, pool_worker, &job) == 0) ++started;
    pool_worker(&job);
    for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------------ */
/* Varlen segment lookup.                                                    */
/* Reference: infllmv2_attn_stage1_triton_v2.py:55-64 (and the same scan in  */
/* max_pooling_1d_varlen.py:72-80): a linear scan over all sequences where   */
/* the LAST sequence whose [qs, qe) range holds the token wins; a token that */
/* no sequence holds keeps the zero defaults.                                */
/* ------------------------------------------------------------------------ */
static int find_seq(const int32_t *cu_q, int64_t n_seq, int64_t t) {
    int found = -1;
    for (int64_t b = 0; b < n_seq; ++b)
        if (t >= cu_q[b] && t < cu_q[b + 1]) found = (int)b;
    return found;
}

/* Number of visible compressed keys for a query.
 * Reference: infllmv2_attn_stage1_triton_v2.py:69-72.  Triton's // on signed
 * integers truncates toward zero (semantic.py lowers it to an sdiv), which is
 * C's / as well: for local_q < 15 the first term is 0, not -1. */
int64_t oracle_stage1_visible(int64_t local_q, int64_t q_len, int64_t k_len, int causal) {
    if (!causal) return k_len;
    int64_t off = (local_q - 15) / 16 + k_len - (q_len - 16 + 1) / 16;
    if (off < 0) off = 0;
    if (off > k_len) off = k_len;
    return off;
}

/* ------------------------------------------------------------------------ */
/* Stage 1: compressed-key GQA attention scores summed per head group.      */
/* Reference: infllmv2_attn_stage1_triton_v2.py:19-150 (kernel) and         */
/* :153-228 (wrapper).                                                      */
/*   q   : [T, Hq, D]  values of the bf16 input, widened to float           */
/*   k   : [Tk, Hk, D] values of the bf16 input, widened to float           */
/*   out : [Hk, t_end - t_begin, out_stride] float: the rows of tokens      */
/*         t_begin..t_end-1, fully written (zeros where the reference       */
/*         leaves its torch.zeros fill or maps NaN to 0).                    */
/* Per (kv head g, token t): scores s_hj = (q_h . k_j) * scale for the      */
/* visible keys j, softmax per head h of the group, then the sum over the   */
/* group's heads (:160-161).  Invisible keys and keys past k_len give 0.     */
/* ------------------------------------------------------------------------ */
typedef struct {
    const float *q, *k;
    int64_t T, Hq, Hk, D, n_seq, out_stride, t_begin, nt;
    const int32_t *cu_q, *cu_k;
    float scale;
    int causal;
    float *out;
} stage1_ctx;

static void stage1_rows(int64_t rb, int64_t re, void *vctx) {
    const stage1_ctx *c = (const stage1_ctx *)vctx;
    const int64_t G = c->Hq / c->Hk, D = c->D, Hk = c->Hk, Hq = c->Hq;
    float *s = NULL;
    int64_t s_cap = 0;
    for (int64_t r = rb; r < re; ++r) {
        int64_t g = r / c->nt, t = c->t_begin + r % c->nt;
        float *orow = c->out + (g * c->nt + (t - c->t_begin)) * c->out_stride;
        memset(orow, 0, sizeof(float) * (size_t)c->out_stride);
        int b = find_seq(c->cu_q, c->n_seq, t);
        if (b < 0) continue;
        int64_t local_q = t - c->cu_q[b];
        int64_t q_len = c->cu_q[b + 1] - c->cu_q[b];
        int64_t k_start = c->cu_k[b];
        int64_t k_len = c->cu_k[b + 1] - c->cu_k[b];
        if (k_len <= 0) continue; /* :83-84 */
        int64_t vis = oracle_stage1_visible(local_q, q_len, k_len, c->causal);
        if (vis <= 0) continue; /* empty softmax: NaN in the reference, mapped to 0 */
        /* Columns past the row (a caller-supplied max_seqlen_k smaller than a
         * real k_len) are not written; the softmax still spans every visible
         * key. */
        int64_t wlim = vis < c->out_stride ? vis : c->out_stride;
        if (s_cap < vis) {
            free(s);
            s = (float *)malloc(sizeof(float) * (size_t)vis);
            s_cap = vis;
        }
        for (int64_t h = 0; h < G; ++h) {
            const float *qv = c->q + (t * Hq + g * G + h) * D;
            float m = -INFINITY;
            for (int64_t j = 0; j < vis; ++j) {
                const float *kv = c->k + ((k_start + j) * Hk + g) * D;
                float acc = 0.f;
                for (int64_t d = 0; d < D; ++d) acc += qv[d] * kv[d];
                s[j] = acc * c->scale;
                if (s[j] > m) m = s[j];
            }
            float l = 0.f;
            for (int64_t j = 0; j < vis; ++j) {
                s[j] = expf(s[j] - m);
                l += s[j];
            }
            float inv = 1.f / l;
            for (int64_t j = 0; j < wlim; ++j) orow[j] += s[j] * inv;
        }
        for (int64_t j = 0; j < wlim; ++j)
            if (isnan(orow[j])) orow[j] = 0.f; /* :227 */
    }
    free(s);
}

void oracle_stage1(const float *q, const float *k, int64_t T, int64_t Hq, int64_t Hk,
                   int64_t D, const int32_t *cu_q, const int32_t *cu_k, int64_t n_seq,
                   float scale, int causal, int64_t out_stride, int64_t t_begin,
                   int64_t t_end, float *out) {
    if (t_end > T) t_end = T;
    if (t_begin < 0) t_begin = 0;
    if (t_end <= t_begin || Hk <= 0) return;
    stage1_ctx c = {q, k, T, Hq, Hk, D, n_seq, out_stride, t_begin, t_end - t_begin,
                    cu_q, cu_k, scale, causal, out};
    parallel_for(Hk * c.nt, 4, stage1_rows, &c);
}

/* ------------------------------------------------------------------------ */
/* Max-pooling of compressed scores into sparse blocks.                      */
/* Reference: max_pooling_1d_varlen.py:33-124 (kernel), :127-183 (wrapper).  */
/* The input is read as a flat buffer indexed h*T*fs + t*fs + c with        */
/* fs = max_seqlen_q // stride (:82, :146), whatever its real row length.   */
/* Elements whose flat index falls outside the buffer (in_numel) are        */
/* treated as masked; the reference reads past its allocation there.       */
/* ------------------------------------------------------------------------ */
typedef struct {
    const float *in;
    int64_t in_numel, H, T, fs, n_seq, NB, block_size, stride, init_blocks, local_blocks;
    const int32_t *cu_q, *cu_k, *cache_lens;
    float *out;
} pool_ctx;

static void pool_rows(int64_t rb, int64_t re, void *vctx) {
    const pool_ctx *c = (const pool_ctx *)vctx;
    const int64_t sp = c->block_size / c->stride; /* :144 */
    const int64_t ksize = sp + 1;                 /* :145 */
    const int64_t pad = 1;                        /* :177 */
    for (int64_t r = rb; r < re; ++r) {
        int64_t h = r / c->T, t = r % c->T;
        int64_t k_len = 0, off_bq = 0;
        for (int64_t b = 0; b < c->n_seq; ++b) { /* :72-80, last hit wins */
            if (t >= c->cu_q[b] && t < c->cu_q[b + 1]) {
                k_len = (int64_t)(c->cu_k[b + 1] - c->cu_k[b]) + c->cache_lens[b];
                off_bq = (t - c->cu_q[b]) / c->block_size;
            }
        }
        int64_t base = h * c->T * c->fs + t * c->fs; /* :82 */
        float *orow = c->out + r * c->NB;
        for (int64_t j = 0; j < c->NB; ++j) {
            int64_t ws = j * sp - pad; /* :84 */
            float mx = -INFINITY;
            for (int64_t ki = 0; ki < ksize; ++ki) { /* :88-106 */
                int64_t kp = ws + ki;
                if (kp < 0 || kp >= k_len) continue;
                int64_t off = base + kp;
                if (off < 0 || off >= c->in_numel) continue;
                mx = fmaxf(mx, c->in[off]); /* NaN-ignoring max, like tl.maximum */
            }
            int mask_inf =
                (j < c->init_blocks) || (off_bq >= j && off_bq <= j + c->local_blocks);
            int64_t wlo = ws > 0 ? ws : 0;
            int64_t whi = ws + ksize < k_len ? ws + ksize : k_len;
            int has_window = whi > wlo; /* :112-114 */
            orow[j] = mask_inf ? INFINITY : (has_window ? mx : -INFINITY); /* :116 */
        }
    }
}

void oracle_max_pool(const float *in, int64_t in_numel, int64_t H, int64_t T, int64_t fs,
                     const int32_t *cu_q, const int32_t *cu_k, const int32_t *cache_lens,
                     int64_t n_seq, int64_t NB, int64_t block_size, int64_t stride,
                     int64_t init_blocks, int64_t local_blocks, float *out) {
    pool_ctx c = {in,  in_numel, H,    T,    fs,   n_seq,      NB, block_size, stride,
                  init_blocks, local_blocks, cu_q, cu_k, cache_lens, out};
    parallel_for(H * T, 64, pool_rows, &c);
}

/* ------------------------------------------------------------------------ */
/* Top-k block selection.  The reference has no top-k of its own (its       */
/* caller uses torch.topk); this defines the selection the GPU kernel must  */
/* reproduce exactly:                                                        */
/*   - candidates are the entries that are neither -inf (a block with no    */
/*     compressed keys under it) nor NaN;                                    */
/*   - order by (score descending, block index ascending), keep the first   */
/*     min(K, #candidates);                                                  */
/*   - emit the kept indices in ascending order, then -1 padding.           */
/* The sorted, padded layout mirrors the reference's own top-k fixtures     */
/* (test/test_sparse_kernel.py:80-87).                                      */
/* ------------------------------------------------------------------------ */
typedef struct {
    float v;
    int32_t i;
} vi_t;

static int cmp_vi(const void *a, const void *b) {
    const vi_t *x = (const vi_t *)a, *y = (const vi_t *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

static int cmp_i32(const void *a, const void *b) {
    int32_t x = *(const int32_t *)a, y = *(const int32_t *)b;
    return (x > y) - (x < y);
}

typedef struct {
    const float *in;
    int64_t NB, K;
    int32_t *out;
} topk_ctx;

static void topk_rows(int64_t rb, int64_t re, void *vctx) {
    const topk_ctx *c = (const topk_ctx *)vctx;
    vi_t *buf = (vi_t *)malloc(sizeof(vi_t) * (size_t)(c->NB > 0 ? c->NB : 1));
    for (int64_t r = rb; r < re; ++r) {
        const float *row = c->in + r * c->NB;
        int64_t n = 0;
        for (int64_t j = 0; j < c->NB; ++j) {
            float v = row[j];
            if (isnan(v) || (isinf(v) && v < 0)) continue;
            buf[n].v = v;
            buf[n].i = (int32_t)j;
            ++n;
        }
        qsort(buf, (size_t)n, sizeof(vi_t), cmp_vi);
        int64_t keep = n < c->K ? n : c->K;
        int32_t *orow = c->out + r * c->K;
        for (int64_t s = 0; s < keep; ++s) orow[s] = buf[s].i;
        qsort(orow, (size_t)keep, sizeof(int32_t), cmp_i32);
        for (int64_t s = keep; s < c->K; ++s) orow[s] = -1;
    }
    free(buf);
}

void oracle_topk(const float *in, int64_t rows, int64_t NB, int64_t K, int32_t *out) {
    topk_ctx c = {in, NB, K, out};
    parallel_for(rows, 64, topk_rows, &c);
}

/* ------------------------------------------------------------------------ */
/* Logical top-k block -> physical KV slot ids.                              */
/* Reference: get_table_torch.py:4-44 (get_block_table_ref_torch).          */
/*   out[t, h, k*64 + i] = head_group * block_table[bs, clamp(pos,0,L-1)] + h */
/*   with pos = topk[h,t,k]*64 + i and bs = token_to_bs[t], when             */
/*   pos >= 0 && pos < seqlen[bs] && pos < token_pos_in_bs[t]; else 0.       */
/* head_group is 2 in the torch reference (:12) and H in the Triton kernels  */
/* (get_table_triton.py:252); the two agree for the 2-kv-head model.        */
/* pos_scalar / seqlen_scalar mirror the numel()==1 broadcast (:26).         */
/* Arithmetic is int32 with wrap-around, like the torch int32 tensors.       */
/* ------------------------------------------------------------------------ */
typedef struct {
    const int32_t *topk, *table, *token_to_bs, *pos_in_bs, *seqlen;
    int64_t H, T, K, L;
    int pos_scalar, seqlen_scalar;
    int32_t head_group;
    int32_t *out;
} gbt_ctx;

static void gbt_rows(int64_t tb, int64_t te, void *vctx) {
    const gbt_ctx *c = (const gbt_ctx *)vctx;
    const int64_t BS = 64; /* kSparseBlockSize, :13 */
    for (int64_t t = tb; t < te; ++t) {
        int32_t bs = c->token_to_bs[t];
        int32_t lim = c->pos_scalar ? c->pos_in_bs[0] : c->pos_in_bs[t];
        int32_t sl = c->seqlen_scalar ? c->seqlen[0] : c->seqlen[bs];
        const int32_t *trow = c->table + (int64_t)bs * c->L;
        for (int64_t h = 0; h < c->H; ++h) {
            for (int64_t kk = 0; kk < c->K; ++kk) {
                int32_t idx = c->topk[(h * c->T + t) * c->K + kk];
                int32_t *o = c->out + (t * c->H + h) * c->K * BS + kk * BS;
                for (int64_t i = 0; i < BS; ++i) {
                    int32_t pos = (int32_t)((uint32_t)idx * (uint32_t)BS + (uint32_t)i);
                    int valid = pos >= 0 && pos < sl && pos < lim; /* :43-54 */
                    int64_t sp = pos < 0 ? 0 : (pos > c->L - 1 ? c->L - 1 : pos); /* :56 */
                    uint32_t v = (uint32_t)c->head_group * (uint32_t)trow[sp] + (uint32_t)h;
                    o[i] = valid ? (int32_t)v : 0; /* :60-63 */
                }
            }
        }
    }
}

void oracle_get_block_table(const int32_t *topk, int64_t H, int64_t T, int64_t K,
                            const int32_t *table, int64_t B, int64_t L,
                            const int32_t *token_to_bs, const int32_t *pos_in_bs,
                            int pos_scalar, const int32_t *seqlen, int seqlen_scalar,
                            int32_t head_group, int32_t *out) {
    (void)B;
    gbt_ctx c = {topk, table, token_to_bs, pos_in_bs, seqlen, H,         T,
                 K,    L,     pos_scalar,  seqlen_scalar,    head_group, out};
    parallel_for(T, 16, gbt_rows, &c);
}

/* ------------------------------------------------------------------ key compression
 * The stage-1 input k_cmp from the keys (no reference code: the reference's
 * caller builds it; the layout follows the 16-token compression stride of
 * infllmv2_attn_stage1_triton_v2.py:70): compressed key j of sequence b is
 * bf16(sum_{t<kernel} k[cu_in[b] + j*stride + t] * (1/kernel)), summed in fp32 in
 * token order, rounded to nearest even; out_bits [cu_out[n_seq], Hk, 128] bf16 bits. */
static uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void oracle_compress_keys(const float *k, int64_t Hk, const int32_t *cu_in, const int32_t *cu_out,
                          int64_t n_seq, int64_t kernel, int64_t stride, uint16_t *out_bits) {
    const float inv = 1.0f / (float)kernel;
    for (int64_t b = 0; b < n_seq; ++b) {
        for (int64_t j = 0; j < (int64_t)cu_out[b + 1] - cu_out[b]; ++j) {
            const int64_t t0 = (int64_t)cu_in[b] + j * stride;
            for (int64_t h = 0; h < Hk; ++h) {
                for (int64_t d = 0; d < 128; ++d) {
                    float acc = 0.f;
                    for (int64_t t = 0; t < kernel; ++t) acc += k[((t0 + t) * Hk + h) * 128 + d];
                    out_bits[(((int64_t)cu_out[b] + j) * Hk + h) * 128 + d] = f32_to_bf16_rne(acc * inv);
                }
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Stage-2 sparse attention over the selected blocks: the consumer of       */
/* get_block_table (no reference implementation; the definition follows the */
/* slot rule of get_table_torch.py:29-44).  For token t, kv head g and each */
/* query head h of the group g*G .. g*G+G-1:                                 */
/*   positions p = topk[g,t,k]*64 + i (k < K, i < 64) with topk >= 0,        */
/*   p < seqlen_q[bs] and p < token_pos_in_bs[t] (bs = token_to_bs[t]);       */
/*   slot_p = head_group * block_table[bs, clamp(p, 0, L-1)] + g;             */
/*   out[t,h] = sum_p softmax_p(q[t,h] . kc[slot_p] * scale) * vc[slot_p],    */
/* in double accumulators, 0 when no position is valid.                      */
/* ------------------------------------------------------------------------ */
typedef struct {
    const float *q, *kc, *vc;
    const int32_t *topk, *table, *tb, *pos, *seqlen;
    int64_t T, Hq, Hk, D, K, L, n_slots;
    int32_t head_group;
    float scale;
    float *out;
} sattn_ctx;

static void sattn_rows(int64_t rb, int64_t re, void *vctx) {
    const sattn_ctx *c = (const sattn_ctx *)vctx;
    const int64_t G = c->Hq / c->Hk, npos = c->K * 64;
    int64_t *slot = (int64_t *)malloc(sizeof(int64_t) * (size_t)(npos > 0 ? npos : 1));
    double *s = (double *)malloc(sizeof(double) * (size_t)(npos > 0 ? npos : 1));
    double *acc = (double *)malloc(sizeof(double) * (size_t)c->D);
    for (int64_t r = rb; r < re; ++r) {
        const int64_t t = r / c->Hk, g = r % c->Hk;
        const int64_t bs = c->tb[t];
        int64_t n = 0;
        for (int64_t k = 0; k < c->K; ++k) {
            const int32_t blk = c->topk[(g * c->T + t) * c->K + k];
            if (blk < 0) continue;
            for (int64_t i = 0; i < 64; ++i) {
                const int64_t p = (int64_t)blk * 64 + i;
                if (p >= c->seqlen[bs] || p >= c->pos[t]) continue;
                const int64_t col = p < 0 ? 0 : (p > c->L - 1 ? c->L - 1 : p);
                const int64_t sl = (int64_t)c->head_group * c->table[bs * c->L + col] + g;
                if (sl < 0 || sl >= c->n_slots) continue; /* outside the cache: not a valid key */
                slot[n++] = sl;
            }
        }
        for (int64_t hh = 0; hh < G; ++hh) {
            const int64_t h = g * G + hh;
            float *o = c->out + (t * c->Hq + h) * c->D;
            const float *qr = c->q + (t * c->Hq + h) * c->D;
            if (n == 0) {
                for (int64_t d = 0; d < c->D; ++d) o[d] = 0.f;
                continue;
            }
            double m = -INFINITY;
            for (int64_t j = 0; j < n; ++j) {
                const float *kr = c->kc + slot[j] * c->D;
                double dot = 0.0;
                for (int64_t d = 0; d < c->D; ++d) dot += (double)qr[d] * (double)kr[d];
                s[j] = dot * (double)c->scale;
                if (s[j] > m) m = s[j];
            }
            double l = 0.0;
            for (int64_t d = 0; d < c->D; ++d) acc[d] = 0.0;
            for (int64_t j = 0; j < n; ++j) {
                const double e = exp(s[j] - m);
                l += e;
                const float *vr = c->vc + slot[j] * c->D;
                for (int64_t d = 0; d < c->D; ++d) acc[d] += e * (double)vr[d];
            }
            for (int64_t d = 0; d < c->D; ++d) o[d] = (float)(acc[d] / l);
        }
    }
    free(slot);
    free(s);
    free(acc);
}

void oracle_sparse_attn(const float *q, int64_t T, int64_t Hq, int64_t D, const float *kc,
                        const float *vc, int64_t n_slots, int64_t Hk, const int32_t *topk, int64_t K,
                        const int32_t *table, int64_t B, int64_t L, const int32_t *token_to_bs,
                        const int32_t *pos_in_bs, const int32_t *seqlen, int32_t head_group,
                        float scale, float *out) {
    (void)B;
    sattn_ctx c = {q, kc, vc, topk, table, token_to_bs, pos_in_bs, seqlen, T, Hq, Hk, D, K, L,
                   n_slots, head_group, scale, out};
    parallel_for(T * Hk, 8, sattn_rows, &c);
}
