// internal.h - helpers shared by the translation units of libemmy_launch.so (not part of the C ABI).
#ifndef EMMY_INTERNAL_H
#define EMMY_INTERNAL_H

// Records the message for emmy_last_error() on this thread and returns `code`.
int emmy_internal_fail(int code, const char* fmt, ...);

// Makes the context selected by emmy_init() current on this thread (EMMY_ERR_NOT_INIT when there is
// none) and, if context_id is non-null, stores an identifier of that context that stays unique
// for the process's lifetime (cuCtxGetId where the driver has it).
int emmy_internal_ready(unsigned long long* context_id);

#endif
