/* Declarations of the part of R's C API that jaxr_b200/r/jxrng_r.c uses, so that the
 * shim's R glue can be compile-checked where R is not installed.  Names and signatures
 * are R's public API (R.h, Rinternals.h, R_ext/Rdynload.h); nothing here is R itself. */
#ifndef JXR_TEST_R_H
#define JXR_TEST_R_H
#include <stddef.h>
char* R_alloc(size_t nelem, int eltsize);
void Rf_error(const char* fmt, ...) __attribute__((noreturn));
#endif
