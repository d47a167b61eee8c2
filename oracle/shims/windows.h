/* Linux stand-in for the handful of Win32 loader calls ds_forward.cpp makes
 * (it opens its sibling fp8_linear library at run time).
 *
 * Test infrastructure only (oracle/Makefile -> oracle/_ref/).  The calls map
 * onto dladdr/dlopen/dlsym; the sibling is looked up next to this library
 * under the same "*.dll" file name the reference expects.
 */
#pragma once
#include <dlfcn.h>
#include <string.h>

typedef void* HMODULE;
typedef const char* LPCSTR;
typedef unsigned long DWORD;
typedef int BOOL;

#ifndef MAX_PATH
#define MAX_PATH 4096
#endif
#define GET_MODULE_HANDLE_EX_FLAG_FROM_ADDRESS 0x4
#define GET_MODULE_HANDLE_EX_FLAG_UNCHANGED_REFCOUNT 0x2

/* The "module handle" of an address is the path of the object containing it;
 * GetModuleFileNameA copies that path out again. */
static inline BOOL GetModuleHandleExA(DWORD flags, LPCSTR address, HMODULE* out) {
    (void)flags;
    Dl_info info;
    if (dladdr((const void*)address, &info) == 0 || info.dli_fname == NULL) {
        return 0;
    }
    *out = (HMODULE)info.dli_fname;
    return 1;
}

static inline DWORD GetModuleFileNameA(HMODULE module, char* path, DWORD size) {
    const char* name = (const char*)module;
    if (name == NULL || size == 0) {
        return 0;
    }
    strncpy(path, name, size - 1);
    path[size - 1] = '\0';
    return (DWORD)strlen(path);
}

static inline HMODULE LoadLibraryA(const char* name) {
    return dlopen(name, RTLD_NOW | RTLD_LOCAL);
}

static inline void* GetProcAddress(HMODULE module, const char* symbol) {
    return dlsym(module, symbol);
}
