// internal.h - helpers shared by the translation units of libemmy_launch.so (not part of the C ABI).
#ifndef EMMY_INTERNAL_H
#define EMMY_INTERNAL_H

// Records the message for emmy_last_error() on this thread and returns `code`.
int emmy_internal_fail(int code, const char* fmt, ...);

#endif
