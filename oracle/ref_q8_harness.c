/*
 * TEST INFRASTRUCTURE (oracle) -- never linked into the product library.
 *
 * Runs the reference's Qwen2.5-0.5B LM-head kernel,
 * compute/gguf-real-weights-loader/kernel_q8_0.cl (gemv_q8_0, :10-61), on the
 * CPU: the OpenCL C source is compiled unmodified as C (the Makefile passes
 * its path as REF_Q8_SRC) under a few definitions of the OpenCL names it uses,
 * and every work-group is executed by a small scheduler that runs its 128
 * work-items as coroutines (ucontext), switching at each barrier():
 *
 *   - __kernel, __global  vanish; __local becomes `static volatile`, so the
 *     work-group's sh_red[128] is one array shared by its work-items (one
 *     group runs at a time) and is re-read after every barrier;
 *   - get_local_id(0) / get_group_id(0) return the running work-item's ids;
 *   - barrier() parks the work-item; the scheduler resumes each work-item in
 *     turn until every one has reached the barrier, then releases them;
 *   - vload_half() converts an IEEE binary16 value exactly to float;
 *   - uchar, ushort and char (signed, -fsigned-char) keep their OpenCL widths.
 *
 * The reference has no CPU path for this kernel (its host program only
 * enqueues it, generate_stream_05b.c:643-664, :845-864), so this is the only
 * way to run its own arithmetic here.  Exported:
 *   ref_gemv_q8_0(W, x, y, M, K)  y[r] for r < M, groups of 4 rows as the
 *                                 host enqueues them (global = ceil(M/4)*128).
 */
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <ucontext.h>

typedef unsigned char uchar;
typedef unsigned short ushort;
typedef unsigned int uint;

#define __kernel
#define __global
#define __local static volatile
#define CLK_LOCAL_MEM_FENCE 1
#define reqd_work_group_size(x, y, z) unused

#define Q8_WG 128

static int q8_cur;      /* running work-item */
static int q8_group;    /* running work-group */

static size_t get_local_id(int dim) { return dim == 0 ? (size_t)q8_cur : 0; }
static size_t get_group_id(int dim) { return dim == 0 ? (size_t)q8_group : 0; }

static float q8_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0x1Fu) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {  /* subnormal: normalise */
        exp = 113;
        while (!(man & 0x400u)) {
            man <<= 1;
            exp--;
        }
        bits = sign | (exp << 23) | ((man & 0x3FFu) << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

static float vload_half(size_t offset, const ushort *p) { return q8_half_to_float(p[offset]); }

static void barrier(int flags);

#include REF_Q8_SRC

/* ---- the work-group scheduler ---- */
static ucontext_t q8_sched;
static ucontext_t q8_ctx[Q8_WG];
static int q8_parked[Q8_WG];  /* 1: at a barrier, 2: returned */
static char *q8_stacks;
static const uchar *q8_W;
static const float *q8_x;
static float *q8_y;
static int q8_M, q8_K;

static void barrier(int flags) {
    (void)flags;
    q8_parked[q8_cur] = 1;
    swapcontext(&q8_ctx[q8_cur], &q8_sched);
}

static void q8_entry(void) {
    gemv_q8_0(q8_W, q8_x, q8_y, q8_M, q8_K);
    q8_parked[q8_cur] = 2;
    /* uc_link returns to the scheduler */
}

#define Q8_STACK (64 * 1024)

int ref_gemv_q8_0(const uint8_t *W, const float *x, float *y, int M, int K) {
    if (!q8_stacks) {
        q8_stacks = (char *)malloc((size_t)Q8_WG * Q8_STACK);
        if (!q8_stacks) return -1;
    }
    q8_W = W;
    q8_x = x;
    q8_y = y;
    q8_M = M;
    q8_K = K;
    const int groups = (M + 3) / 4;
    for (int g = 0; g < groups; g++) {
        q8_group = g;
        for (int i = 0; i < Q8_WG; i++) {
            if (getcontext(&q8_ctx[i]) != 0) return -1;
            q8_ctx[i].uc_stack.ss_sp = q8_stacks + (size_t)i * Q8_STACK;
            q8_ctx[i].uc_stack.ss_size = Q8_STACK;
            q8_ctx[i].uc_link = &q8_sched;
            makecontext(&q8_ctx[i], q8_entry, 0);
            q8_parked[i] = 0;
        }
        /* Each pass resumes every live work-item until it parks at the next
         * barrier or returns; the kernel's barriers are reached by all 128. */
        for (;;) {
            int live = 0;
            for (int i = 0; i < Q8_WG; i++) {
                if (q8_parked[i] == 2) continue;
                q8_cur = i;
                q8_parked[i] = 0;
                if (swapcontext(&q8_sched, &q8_ctx[i]) != 0) return -1;
                if (q8_parked[i] != 2) live++;
            }
            if (!live) break;
        }
    }
    return 0;
}
