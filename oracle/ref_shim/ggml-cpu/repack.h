/*
 * Stand-in for ggml-cpu/repack.h, holding only the four block layouts that the
 * reference's tools/trace/exact_packed_cpu.h uses, so that header compiles
 * without a llama.cpp checkout.  The layouts are ggml's on-disk / repacked
 * formats (an interface that has to match byte for byte):
 *   block_q8_0    = { fp16 d; int8 qs[32]; }            34 bytes
 *   block_mxfp4   = { uint8 e; uint8 qs[16]; }          17 bytes
 *   block_mxfp4x8 = { uint8 e[8]; uint8 qs[128]; }      eight rows, 8-byte interleave
 *   block_q8_0x4  = { fp16 d[4]; int8 qs[128]; }        four rows, 8-byte interleave
 * Test infrastructure only (used by oracle/ref_wrap.cpp).
 */
#pragma once
#include <cstdint>

typedef uint16_t ggml_half;

struct block_q8_0 {
    ggml_half d;
    int8_t qs[32];
};

struct block_mxfp4 {
    uint8_t e;
    uint8_t qs[16];
};

struct block_mxfp4x8 {
    uint8_t e[8];
    uint8_t qs[128];
};

struct block_q8_0x4 {
    ggml_half d[4];
    int8_t qs[128];
};

static_assert(sizeof(block_q8_0) == 34, "block_q8_0 layout");
static_assert(sizeof(block_mxfp4) == 17, "block_mxfp4 layout");
static_assert(sizeof(block_mxfp4x8) == 136, "block_mxfp4x8 layout");
static_assert(sizeof(block_q8_0x4) == 136, "block_q8_0x4 layout");
