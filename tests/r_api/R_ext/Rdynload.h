/* See R.h one directory up: declarations only, for compile-checking the shim's R glue. */
#ifndef JXR_TEST_RDYNLOAD_H
#define JXR_TEST_RDYNLOAD_H
#include "../Rinternals.h"
typedef void* (*DL_FUNC)(void);
typedef struct {
  const char* name;
  DL_FUNC fun;
  int numArgs;
} R_CallMethodDef;
typedef struct _DllInfo DllInfo;
int R_registerRoutines(DllInfo* info, const void* c_routines, const R_CallMethodDef* call_routines,
                       const void* fortran_routines, const void* external_routines);
Rboolean R_useDynamicSymbols(DllInfo* info, Rboolean value);
#endif
