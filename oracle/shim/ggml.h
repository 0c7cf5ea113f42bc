// Test-infrastructure shim (oracle only, never linked into the product): the handful of ggml names
// that the reference's host-side planner source (src/hjepa-plan.cpp and the headers it includes)
// uses, written from those call sites -- a tensor record with a type and four extents, element and
// byte counts, the f16 row conversion and the dequantisation trait of the block formats. No ggml
// source exists in this tree or on this machine; nothing here comes from it.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

typedef uint16_t ggml_fp16_t;

enum ggml_type {
    GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q4_0 = 2, GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6, GGML_TYPE_Q5_1 = 7, GGML_TYPE_Q8_0 = 8, GGML_TYPE_BF16 = 30,
};

struct ggml_context;
struct ggml_cgraph;

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    int     n_dims;
    size_t  nbytes;
    void *  data;        // host bytes in the file's own encoding
};

#define GGML_RESTRICT __restrict__
#define GGML_ASSERT(x) do { if (!(x)) { fprintf(stderr, "GGML_ASSERT(%s) failed at %s:%d\n", #x, __FILE__, __LINE__); abort(); } } while (0)

int64_t ggml_nelements(const struct ggml_tensor * t);
size_t  ggml_nbytes(const struct ggml_tensor * t);
int     ggml_n_dims(const struct ggml_tensor * t);
void    ggml_fp16_to_fp32_row(const ggml_fp16_t * x, float * y, int64_t n);

typedef void (*ggml_to_float_t)(const void * x, float * y, int64_t k);
struct ggml_type_traits {
    const char *    type_name;
    int64_t         blck_size;
    size_t          type_size;
    ggml_to_float_t to_float;
};
const struct ggml_type_traits * ggml_get_type_traits(enum ggml_type type);
