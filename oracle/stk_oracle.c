/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the streaming top-k SAE encoder.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * this library, and only as the checker.  The product path (the sm_100a CUDA
 * library under streamtopk-sae_b200/) never calls it.
 *
 * This is a plain-C restatement of the reference's CPU algorithm
 *   streamtopk_sae/csrc/cpu/streamtopk_cpu.cpp:15-67   (process_row<K>)
 *   streamtopk_sae/csrc/cpu/streamtopk_cpu.cpp:70-79   (dispatch_rows<K>, serial rows)
 *   streamtopk_sae/csrc/cpu/topk_buffer.hpp:9-72       (TopKBuffer<K>, heap when K > 64)
 * restated without libtorch:
 *   - F is walked in tiles of 512 features (streamtopk_cpu.cpp:12,33-35);
 *   - each score is accumulated in fp32, bias first, then x[dd]*w[f][dd] in
 *     increasing dd (streamtopk_cpu.cpp:39-46);
 *   - a score enters the buffer only if it is strictly greater than the
 *     current threshold (streamtopk_cpu.cpp:49-55, topk_buffer.hpp:30,42);
 *   - the buffer starts at (-inf, -1) (topk_buffer.hpp:13-18);
 *   - K <= 64 keeps a descending insertion-sorted array, K > 64 a binary
 *     min-heap whose root is the minimum (topk_buffer.hpp:9, 29-60);
 *   - the output is the buffer in its own order: descending for K <= 64,
 *     heap order for K > 64 (streamtopk_cpu.cpp:58-66).
 * Unlike the reference, any 1 <= k <= F is accepted (the reference only
 * instantiates k in {1,2,4,8,16,32,64,128}, streamtopk_cpu.cpp:110-122);
 * the heap/insertion choice follows the same K > 64 rule.
 *
 * Build: oracle/Makefile (plain gcc, -O2, no fast-math, so the fp32
 * accumulation order is exactly the sequential one written here).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define STK_ORACLE_TILE 512

typedef struct {
    float* values;
    int32_t* indices;
    int64_t K;
    int use_heap;
} topk_buf;

static void buf_init(topk_buf* b) {
    for (int64_t i = 0; i < b->K; ++i) {
        b->values[i] = -INFINITY;
        b->indices[i] = -1;
    }
}

static float buf_threshold(const topk_buf* b) {
    return b->use_heap ? b->values[0] : b->values[b->K - 1];
}

static void buf_try_insert(topk_buf* b, float v, int32_t idx) {
    const int64_t K = b->K;
    float* vals = b->values;
    int32_t* ids = b->indices;
    if (!b->use_heap) {
        if (v <= vals[K - 1]) return;
        int64_t pos = K - 1;
        while (pos > 0 && vals[pos - 1] < v) {
            vals[pos] = vals[pos - 1];
            ids[pos] = ids[pos - 1];
            --pos;
        }
        vals[pos] = v;
        ids[pos] = idx;
    } else {
        if (v <= vals[0]) return;
        vals[0] = v;
        ids[0] = idx;
        int64_t i = 0;
        for (;;) {
            int64_t l = 2 * i + 1, r = 2 * i + 2, s = i;
            if (l < K && vals[l] < vals[s]) s = l;
            if (r < K && vals[r] < vals[s]) s = r;
            if (s == i) break;
            float tv = vals[i]; vals[i] = vals[s]; vals[s] = tv;
            int32_t ti = ids[i]; ids[i] = ids[s]; ids[s] = ti;
            i = s;
        }
    }
}

/* Streaming top-k of one row (restates process_row<K>). */
static void process_row(const float* xi, const float* W, const float* bias,
                        int64_t d, int64_t F, topk_buf* buf, float* scores) {
    for (int64_t f0 = 0; f0 < F; f0 += STK_ORACLE_TILE) {
        int64_t f_end = f0 + STK_ORACLE_TILE < F ? f0 + STK_ORACLE_TILE : F;
        int64_t tile = f_end - f0;
        for (int64_t j = 0; j < tile; ++j) {
            const float* wj = W + (f0 + j) * d;
            float s = bias[f0 + j];
            for (int64_t dd = 0; dd < d; ++dd) s += xi[dd] * wj[dd];
            scores[j] = s;
        }
        float thr = buf_threshold(buf);
        for (int64_t j = 0; j < tile; ++j) {
            if (scores[j] > thr) {
                buf_try_insert(buf, scores[j], (int32_t)(f0 + j));
                thr = buf_threshold(buf);
            }
        }
    }
}

/*
 * X (B,d) fp32 row-major, W (F,d) fp32 row-major, bias (F,) fp32.
 * Writes V (B,k) fp32 and I (B,k) int32 in buffer order.
 * Rows [row_begin, row_end) only, so callers can shard rows over processes.
 * Returns 0 on success, 1 on bad arguments, 2 on allocation failure.
 */
int stk_oracle_stream_topk(const float* X, const float* W, const float* bias,
                           float* V, int32_t* I, int64_t B, int64_t d,
                           int64_t F, int64_t k, int64_t row_begin,
                           int64_t row_end) {
    if (B < 0 || d < 1 || F < 1 || k < 1 || k > F) return 1;
    if (row_begin < 0 || row_end > B || row_begin > row_end) return 1;
    float* vals = (float*)malloc(sizeof(float) * (size_t)k);
    int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)k);
    float* scores = (float*)malloc(sizeof(float) * STK_ORACLE_TILE);
    if (!vals || !ids || !scores) {
        free(vals); free(ids); free(scores);
        return 2;
    }
    topk_buf buf = {vals, ids, k, k > 64};
    for (int64_t i = row_begin; i < row_end; ++i) {
        buf_init(&buf);
        process_row(X + i * d, W, bias, d, F, &buf, scores);
        memcpy(V + i * k, vals, sizeof(float) * (size_t)k);
        memcpy(I + i * k, ids, sizeof(int32_t) * (size_t)k);
    }
    free(vals); free(ids); free(scores);
    return 0;
}

/*
 * Dense fp64 scores of rows [row_begin,row_end) against features [f_begin,f_end):
 * S[(i-row_begin)*(f_end-f_begin) + (f-f_begin)] = bias[f] + sum_dd X[i,dd]*W[f,dd]
 * in double precision.  Used as the "true score" reference for tie-aware checks.
 */
int stk_oracle_scores_f64(const float* X, const float* W, const float* bias,
                          double* S, int64_t d, int64_t row_begin,
                          int64_t row_end, int64_t f_begin, int64_t f_end) {
    if (d < 1 || row_begin > row_end || f_begin > f_end) return 1;
    const int64_t nf = f_end - f_begin;
    for (int64_t i = row_begin; i < row_end; ++i) {
        const float* xi = X + i * d;
        for (int64_t f = f_begin; f < f_end; ++f) {
            const float* wf = W + f * d;
            double s = (double)bias[f];
            for (int64_t dd = 0; dd < d; ++dd) s += (double)xi[dd] * (double)wf[dd];
            S[(i - row_begin) * nf + (f - f_begin)] = s;
        }
    }
    return 0;
}
