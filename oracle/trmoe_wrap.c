/* trmoe_wrap.c: test infrastructure. Linked into a build of Trochilus's own engine (oracle/Makefile, target
 * `engine`) with `-Wl,--wrap=<name>` for every kernel-level function the library replaces, so the unmodified engine
 * (src/models/olmoe.c) runs its matmuls, softmax and SwiGLU on the GPU through libtrmoe.so. This is the relink
 * INTEGRATION.md's section 1 describes, made real for the full-model greedy-token check (tests/test_gpu_engine.py):
 * the same engine with and without the wrap must give the same tokens and the same logits.
 *
 * __wrap_X forwards to the library's X. The two share a name, so the library is opened RTLD_LOCAL and X bound by
 * handle (the engine's own X stays reachable as __real_X, unused here). The library is found at $TRMOE_LIB, else
 * beside this binary's directory at ../../trochilus_b200/libtrmoe.so. A missing library or symbol ends the process:
 * a wrapped engine that silently ran the CPU would make the comparison meaningless.
 *
 * At exit the shim prints `gpu: libtrmoe.so on <device>, <n> kernel-level calls` on stderr: the proof that the
 * GPU ran, as the reference's own GPU gate asks for a `gpu:` line (tools/gpu_exact.sh). */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <limits.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "trmoe.h"

static void *g_lib;
static atomic_ullong g_calls;
static char g_device[128] = "(no device)";

static void report(void) {
    if (g_lib == NULL) return;
    fprintf(stderr, "gpu: libtrmoe.so on %s, %llu kernel-level calls\n", g_device,
            (unsigned long long)atomic_load(&g_calls));
}

/* the device's name, read once when the library is opened (at exit the CUDA runtime may be gone already) */
static void name_device(void) {
    tr_gpu *(*open_fn)(char *, size_t) = (tr_gpu * (*)(char *, size_t)) dlsym(g_lib, "tr_gpu_open");
    const char *(*name_fn)(const tr_gpu *) = (const char *(*)(const tr_gpu *))dlsym(g_lib, "tr_gpu_name");
    void (*close_fn)(tr_gpu *) = (void (*)(tr_gpu *))dlsym(g_lib, "tr_gpu_close");
    char err[128] = "";
    tr_gpu *g = open_fn ? open_fn(err, sizeof err) : NULL;
    if (g != NULL && name_fn != NULL) snprintf(g_device, sizeof g_device, "%s", name_fn(g));
    if (g != NULL && close_fn != NULL) close_fn(g);
}

static void *lib(void) {
    if (g_lib != NULL) return g_lib;
    char path[PATH_MAX + 64];
    const char *env = getenv("TRMOE_LIB");
    if (env != NULL && env[0] != 0) {
        snprintf(path, sizeof path, "%s", env);
    } else {
        char self[PATH_MAX];
        const ssize_t n = readlink("/proc/self/exe", self, sizeof self - 1);
        if (n <= 0) {
            fprintf(stderr, "trmoe_wrap: cannot find this binary's path; set TRMOE_LIB\n");
            exit(70);
        }
        self[n] = 0;
        char *slash = strrchr(self, '/');
        if (slash != NULL) *slash = 0;
        snprintf(path, sizeof path, "%s/../../trochilus_b200/libtrmoe.so", self);
    }
    g_lib = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (g_lib == NULL) {
        fprintf(stderr, "trmoe_wrap: %s\n", dlerror());
        exit(70);
    }
    name_device();
    atexit(report);
    return g_lib;
}

static void *sym(const char *name) {
    void *f = dlsym(lib(), name);
    if (f == NULL) {
        fprintf(stderr, "trmoe_wrap: libtrmoe.so has no %s\n", name);
        exit(70);
    }
    return f;
}

/* one forwarder per wrapped name: the function pointer is bound once, every call counted */
#define FORWARD_VOID(name, params, args)                                                                                \
    void __wrap_##name params {                                                                                        \
        static void(*f) params;                                                                                        \
        if (f == NULL) f = (void(*) params)sym(#name);                                                                 \
        atomic_fetch_add(&g_calls, 1);                                                                                 \
        f args;                                                                                                        \
    }
#define FORWARD_INT(name, params, args)                                                                                 \
    int __wrap_##name params {                                                                                         \
        static int(*f) params;                                                                                         \
        if (f == NULL) f = (int(*) params)sym(#name);                                                                  \
        atomic_fetch_add(&g_calls, 1);                                                                                 \
        return f args;                                                                                                 \
    }

FORWARD_VOID(tr_matmul, (tr_pool * p, const tr_mat *w, const float *x, int64_t n, float *y), (p, w, x, n, y))
FORWARD_VOID(tr_matmul_s, (tr_pool * p, const tr_mat *w, const float *x, int64_t n, float *y, const void *s),
             (p, w, x, n, y, s))
FORWARD_VOID(tr_matmul_grouped,
             (tr_pool * p, const tr_mat *w, const int64_t *off, int64_t ng, const float *x, float *y),
             (p, w, off, ng, x, y))
FORWARD_VOID(tr_matmul_grouped_s,
             (tr_pool * p, const tr_mat *w, const int64_t *off, int64_t ng, const float *x, float *y, const void *s),
             (p, w, off, ng, x, y, s))
FORWARD_VOID(tr_softmax, (float *x, int64_t n), (x, n))
FORWARD_VOID(tr_swiglu, (tr_pool * p, float *x, const float *y, int64_t n), (p, x, y, n))
FORWARD_INT(tr_q4x_road, (tr_pool * p, const tr_mat *w, const int64_t *off, int64_t ng, const void *s),
            (p, w, off, ng, s))
FORWARD_VOID(tr_q4x_prepare, (tr_pool * p, const float *x, int64_t n, int64_t cols, void *xq), (p, x, n, cols, xq))
FORWARD_INT(tr_matmul_q4x_prepared,
            (tr_pool * p, const tr_mat *w, const int64_t *off, int64_t ng, const void *xq, const int64_t *map, float *y,
             const void *s),
            (p, w, off, ng, xq, map, y, s))
FORWARD_INT(tr_matmul_q4x_prepared_n,
            (tr_pool * p, const tr_mat *const *w, int nw, const int64_t *off, int64_t ng, const void *xq,
             const int64_t *map, float *const *y, const void *s),
            (p, w, nw, off, ng, xq, map, y, s))
FORWARD_VOID(tr_swiglu_prepare, (tr_pool * p, float *x, const float *y, int64_t rows, int64_t n, void *xq),
             (p, x, y, rows, n, xq))
