/* POSIX stand-ins for the Win32 kernel32 imports of the reference's
 * decode_kernel.c (src/jouleai/native/decode_kernel.c:33-37, 635-650,
 * 1913-1940), so that the UNMODIFIED reference source builds as a Linux
 * shared object and serves as the CPU oracle and the timed CPU baseline.
 *
 * TEST INFRASTRUCTURE ONLY: nothing in the product links this file.
 *
 *   GetModuleHandleA      -> a non-NULL dummy module handle
 *   GetProcAddress        -> GetProcessHeap/HeapAlloc/HeapFree (calloc/free;
 *                            the reference asks for HEAP_ZERO_MEMORY) and
 *                            WaitOnAddress/WakeByAddressAll (Linux futex on
 *                            the low 32-bit word, so idle pool workers sleep
 *                            instead of spinning)
 *   CreateThread          -> pthread_create (joinable; handle = heap record)
 *   WaitForMultipleObjects-> pthread_join of every handle
 *   SetThreadAffinityMask -> no-op
 */
#define _GNU_SOURCE
#include <limits.h>
#include <linux/futex.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <sys/syscall.h>
#include <time.h>
#include <unistd.h>

static int g_dummy_module;

void* GetModuleHandleA(const char* name) {
    (void)name;
    return &g_dummy_module;
}

static void* shim_GetProcessHeap(void) { return &g_dummy_module; }

static void* shim_HeapAlloc(void* heap, unsigned long flags, unsigned long n) {
    (void)heap;
    (void)flags;
    return calloc(1, n ? n : 1);
}

static int shim_HeapFree(void* heap, unsigned long flags, void* p) {
    (void)heap;
    (void)flags;
    free(p);
    return 1;
}

/* WaitOnAddress(addr, compare, size, ms): sleep while *addr == *compare. */
static unsigned long shim_WaitOnAddress(volatile void* addr, void* compare,
                                        size_t size, unsigned long ms) {
    if (memcmp((const void*)addr, compare, size) != 0) return 1;
    int32_t expect;
    memcpy(&expect, compare, sizeof expect); /* little-endian low word */
    struct timespec ts, *tsp = NULL;
    if (ms != 0xFFFFFFFFul) {
        ts.tv_sec = (time_t)(ms / 1000);
        ts.tv_nsec = (long)(ms % 1000) * 1000000L;
        tsp = &ts;
    }
    syscall(SYS_futex, (int32_t*)addr, FUTEX_WAIT_PRIVATE, expect, tsp, NULL, 0);
    return 1;
}

static unsigned long shim_WakeByAddressAll(volatile void* addr) {
    syscall(SYS_futex, (int32_t*)addr, FUTEX_WAKE_PRIVATE, INT_MAX, NULL, NULL, 0);
    return 0;
}

void* GetProcAddress(void* mod, const char* name) {
    (void)mod;
    if (!strcmp(name, "GetProcessHeap")) return (void*)shim_GetProcessHeap;
    if (!strcmp(name, "HeapAlloc")) return (void*)shim_HeapAlloc;
    if (!strcmp(name, "HeapFree")) return (void*)shim_HeapFree;
    if (!strcmp(name, "WaitOnAddress")) return (void*)shim_WaitOnAddress;
    if (!strcmp(name, "WakeByAddressAll")) return (void*)shim_WakeByAddressAll;
    return NULL;
}

typedef unsigned long (*thread_fn)(void*);
typedef struct {
    pthread_t tid;
    thread_fn fn;
    void* arg;
} shim_thread;

static void* shim_trampoline(void* p) {
    shim_thread* t = (shim_thread*)p;
    t->fn(t->arg);
    return NULL;
}

void* CreateThread(void* sec, size_t stack, thread_fn fn, void* arg,
                   unsigned long flags, unsigned long* id) {
    (void)sec;
    (void)stack;
    (void)flags;
    shim_thread* t = (shim_thread*)calloc(1, sizeof *t);
    if (!t) return NULL;
    t->fn = fn;
    t->arg = arg;
    if (pthread_create(&t->tid, NULL, shim_trampoline, t) != 0) {
        free(t);
        return NULL;
    }
    if (id) *id = (unsigned long)(uintptr_t)t;
    return t;
}

unsigned long WaitForMultipleObjects(unsigned long n, void* const* handles,
                                     int all, unsigned long ms) {
    (void)all;
    (void)ms;
    for (unsigned long i = 0; i < n; i++) {
        shim_thread* t = (shim_thread*)handles[i];
        if (!t) continue;
        pthread_join(t->tid, NULL);
        free(t);
    }
    return 0;
}

void SetThreadAffinityMask(void* h, unsigned long mask) {
    (void)h;
    (void)mask;
}
