/* The part of XLA's FFI C API (API version 0.3) that the jxrng handlers use, declared here
 * so that libjxrng_ffi.so builds without XLA's source tree.
 *
 * This is an ABI: a handler and the XLA runtime that calls it must agree on every struct
 * layout, enum value and table slot below, so the names, field order and values are XLA's
 * own (xla/ffi/api/c_api.h, as vendored by jaxR for ffi_include_dir(), inst/include).
 * Only what the handlers touch is declared: opaque types stay incomplete, and the API
 * function table is declared up to the last slot the handlers read, with later slots
 * left out.  tests/test_ffi_abi.py checks these layouts against XLA's header when one is
 * available ($XLA_FFI_INCLUDE_DIR). */
#ifndef JXRNG_XLA_FFI_ABI_H
#define JXRNG_XLA_FFI_ABI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XLA_FFI_API_MAJOR 0
#define XLA_FFI_API_MINOR 3

/* size of a struct up to and including its last field (every struct carries it) */
#define JXR_FFI_SIZE_UPTO(type, field) (offsetof(type, field) + sizeof(((type*)0)->field))

typedef struct XLA_FFI_Error XLA_FFI_Error;
typedef struct XLA_FFI_ExecutionContext XLA_FFI_ExecutionContext;
typedef struct XLA_FFI_InternalApi XLA_FFI_InternalApi;
typedef struct XLA_FFI_Future XLA_FFI_Future;

typedef enum { XLA_FFI_Extension_Metadata = 1 } XLA_FFI_Extension_Type;

typedef struct XLA_FFI_Extension_Base {
  size_t struct_size;
  XLA_FFI_Extension_Type type;
  struct XLA_FFI_Extension_Base* next;
} XLA_FFI_Extension_Base;

typedef struct XLA_FFI_Api_Version {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  int major_version;
  int minor_version;
} XLA_FFI_Api_Version;

typedef enum {
  XLA_FFI_Error_Code_OK = 0,
  XLA_FFI_Error_Code_INVALID_ARGUMENT = 3,
  XLA_FFI_Error_Code_RESOURCE_EXHAUSTED = 8,
  XLA_FFI_Error_Code_UNIMPLEMENTED = 12,
  XLA_FFI_Error_Code_INTERNAL = 13
} XLA_FFI_Error_Code;

typedef struct XLA_FFI_Error_Create_Args {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  const char* message;
  XLA_FFI_Error_Code errc;
} XLA_FFI_Error_Create_Args;
enum {
  XLA_FFI_Error_Create_Args_STRUCT_SIZE = JXR_FFI_SIZE_UPTO(XLA_FFI_Error_Create_Args, errc)
};

/* element types (xla::PrimitiveType numbering) the handlers accept or produce */
typedef enum {
  XLA_FFI_DataType_INVALID = 0,
  XLA_FFI_DataType_PRED = 1,
  XLA_FFI_DataType_S32 = 4,
  XLA_FFI_DataType_S64 = 5,
  XLA_FFI_DataType_U8 = 6,
  XLA_FFI_DataType_U16 = 7,
  XLA_FFI_DataType_U32 = 8,
  XLA_FFI_DataType_U64 = 9,
  XLA_FFI_DataType_F16 = 10,
  XLA_FFI_DataType_F32 = 11,
  XLA_FFI_DataType_F64 = 12,
  XLA_FFI_DataType_BF16 = 16
} XLA_FFI_DataType;

typedef struct XLA_FFI_Buffer {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  XLA_FFI_DataType dtype;
  void* data;
  int64_t rank;
  int64_t* dims;
} XLA_FFI_Buffer;

typedef enum { XLA_FFI_ArgType_BUFFER = 1 } XLA_FFI_ArgType;
typedef enum { XLA_FFI_RetType_BUFFER = 1 } XLA_FFI_RetType;
typedef enum {
  XLA_FFI_AttrType_ARRAY = 1,
  XLA_FFI_AttrType_DICTIONARY = 2,
  XLA_FFI_AttrType_SCALAR = 3,
  XLA_FFI_AttrType_STRING = 4
} XLA_FFI_AttrType;

typedef struct XLA_FFI_ByteSpan {
  const char* ptr;
  size_t len;
} XLA_FFI_ByteSpan;

typedef struct XLA_FFI_Scalar {
  XLA_FFI_DataType dtype;
  void* value;
} XLA_FFI_Scalar;

typedef struct XLA_FFI_TypeId {
  int64_t type_id;
} XLA_FFI_TypeId;

typedef enum {
  XLA_FFI_ExecutionStage_INSTANTIATE = 0,
  XLA_FFI_ExecutionStage_PREPARE = 1,
  XLA_FFI_ExecutionStage_INITIALIZE = 2,
  XLA_FFI_ExecutionStage_EXECUTE = 3
} XLA_FFI_ExecutionStage;

typedef struct XLA_FFI_Args {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  int64_t size;
  XLA_FFI_ArgType* types;
  void** args;
} XLA_FFI_Args;

typedef struct XLA_FFI_Rets {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  int64_t size;
  XLA_FFI_RetType* types;
  void** rets;
} XLA_FFI_Rets;

typedef struct XLA_FFI_Attrs {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  int64_t size;
  XLA_FFI_AttrType* types;
  XLA_FFI_ByteSpan** names;
  void** attrs;
} XLA_FFI_Attrs;

typedef struct XLA_FFI_Api XLA_FFI_Api;

typedef struct XLA_FFI_CallFrame {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  const XLA_FFI_Api* api;
  XLA_FFI_ExecutionContext* ctx;
  XLA_FFI_ExecutionStage stage;
  XLA_FFI_Args args;
  XLA_FFI_Rets rets;
  XLA_FFI_Attrs attrs;
  XLA_FFI_Future* future;
} XLA_FFI_CallFrame;

typedef uint32_t XLA_FFI_Handler_Traits;

typedef struct XLA_FFI_Stream_Get_Args {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  XLA_FFI_ExecutionContext* ctx;
  void* stream;
} XLA_FFI_Stream_Get_Args;
enum { XLA_FFI_Stream_Get_Args_STRUCT_SIZE = JXR_FFI_SIZE_UPTO(XLA_FFI_Stream_Get_Args, stream) };

typedef struct XLA_FFI_Metadata {
  size_t struct_size;
  XLA_FFI_Api_Version api_version;
  XLA_FFI_Handler_Traits traits;
  XLA_FFI_TypeId state_type_id;
} XLA_FFI_Metadata;

typedef struct XLA_FFI_Metadata_Extension {
  XLA_FFI_Extension_Base extension_base;
  XLA_FFI_Metadata* metadata;
} XLA_FFI_Metadata_Extension;

typedef XLA_FFI_Error* XLA_FFI_Error_Create(XLA_FFI_Error_Create_Args* args);
typedef XLA_FFI_Error* XLA_FFI_Stream_Get(XLA_FFI_Stream_Get_Args* args);

/* The runtime's function table.  Slots the handlers do not call are untyped pointers;
 * the table continues in XLA past XLA_FFI_Stream_Get, and nothing here reads further. */
struct XLA_FFI_Api {
  size_t struct_size;
  XLA_FFI_Extension_Base* extension_start;
  XLA_FFI_Api_Version api_version;
  const XLA_FFI_InternalApi* internal_api;
  XLA_FFI_Error_Create* XLA_FFI_Error_Create;
  void* XLA_FFI_Error_GetMessage;
  void* XLA_FFI_Error_Destroy;
  void* XLA_FFI_Handler_Register;
  XLA_FFI_Stream_Get* XLA_FFI_Stream_Get;
};

#ifdef __cplusplus
}
#endif
#endif /* JXRNG_XLA_FFI_ABI_H */
