/* Shared declarations of the generated tables (cuda target). */
#ifndef NNC_MODEL_TABLES_H
#define NNC_MODEL_TABLES_H
#include <stddef.h>
#include "nnc_types.h"
typedef struct { Tensor* tensor; size_t offset; } nnc_arena_entry;
typedef struct {
    const char* symbol; Tensor* tensor; size_t offset; long long packed_offset;
    size_t packed_bytes; size_t nbytes;
} nnc_const_entry;
extern const size_t nnc_arena_bytes, nnc_const_bytes;
extern const nnc_arena_entry nnc_arena_table[];
extern const int nnc_arena_count;
extern const nnc_const_entry nnc_const_table[];
extern const int nnc_const_count;
extern Tensor* const nnc_input_table[];
extern const int nnc_input_count;
extern Tensor* const nnc_output_table[];
extern const int nnc_output_count;
#endif
