/* See R.h in this directory: declarations only, for compile-checking the shim's R glue. */
#ifndef JXR_TEST_RINTERNALS_H
#define JXR_TEST_RINTERNALS_H
#include <stddef.h>
typedef struct SEXPREC* SEXP;
typedef ptrdiff_t R_xlen_t;
typedef unsigned int SEXPTYPE;
typedef enum { FALSE = 0, TRUE } Rboolean;
#define R_XLEN_T_MAX 4503599627370496
#define LGLSXP 10
#define REALSXP 14
#define VECSXP 19
extern SEXP R_NilValue;
SEXP Rf_allocVector(SEXPTYPE type, R_xlen_t length);
double* REAL(SEXP x);
int* LOGICAL(SEXP x);
R_xlen_t XLENGTH(SEXP x);
int TYPEOF(SEXP x);
SEXP SET_VECTOR_ELT(SEXP x, R_xlen_t i, SEXP v);
SEXP Rf_protect(SEXP s);
void Rf_unprotect(int n);
#define PROTECT(s) Rf_protect(s)
#define UNPROTECT(n) Rf_unprotect(n)
double Rf_asReal(SEXP x);
int Rf_asInteger(SEXP x);
int Rf_asLogical(SEXP x);
#endif
