/*
 * fail_alloc.c — test-only allocation fault injector for the host side.
 * Preloaded (LD_PRELOAD) into a child process, it makes malloc / calloc
 * return NULL for requests of exactly FAIL_ALLOC_SIZE bytes and passes every
 * other request to glibc.  Used to drive train_create's host-allocation
 * failure path; it touches no GPU.
 */
#define _GNU_SOURCE
#include <stddef.h>
#include <stdlib.h>

extern void* __libc_malloc(size_t n);
extern void* __libc_calloc(size_t n, size_t size);

/* Read on every call, so a process can switch the fault off again. */
static size_t fail_size(void) {
    const char* e = getenv("FAIL_ALLOC_SIZE");
    return e ? (size_t)strtoull(e, NULL, 10) : 0;
}

void* malloc(size_t n) {
    if (n != 0 && n == fail_size()) return NULL;
    return __libc_malloc(n);
}

void* calloc(size_t n, size_t size) {
    if (n != 0 && size != 0 && n * size == fail_size()) return NULL;
    return __libc_calloc(n, size);
}
