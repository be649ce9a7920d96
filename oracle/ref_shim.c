/* Test infrastructure: struct sizes of the reference runtime for ctypes callers in tests/ (they allocate a v3_model
 * for v3_load, a v3_governor for the v3_gov_* functions and a v3_tokenizer for v3_encode_ex).  Compiled by oracle/Makefile into
 * oracle/_ref/libvault3.so together with the reference's runtime/vault3.c, against its runtime/vault3.h. */
#include <stddef.h>

#include "vault3.h"

size_t ref_sizeof_model(void) { return sizeof(v3_model); }
size_t ref_sizeof_governor(void) { return sizeof(v3_governor); }
size_t ref_sizeof_tokenizer(void) { return sizeof(v3_tokenizer); }
