/*
 * lalb_c_caller.c -- a plain C99 host program that drives the library the way
 * the reference engine's C sources would: include lalb.h, create a context,
 * hand it device buffers, call the matmul entry points, read the results.
 * No Python and no C++ on this side of the boundary.
 *
 *   lalb_c_caller --abi-only          checks the host-only entry points; a
 *                                     missing sm_100 device is not an error
 *   lalb_c_caller <in.bin> <out.bin>  one Q4_K matvec and one LM-head call
 *
 * in.bin (little-endian): int32 rows, K, head_rows, head_K; then the Q4_K
 * matrix (rows * K/256 * 144 bytes), x (K float32), the int8 LM head
 * (head_rows * head_K bytes), its row scales (head_rows float32) and the
 * LM-head input (head_K float32).
 * out.bin: y (rows float32), logits (head_rows float32), argmax (int32).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "lalb.h"

static int fail(const char *what, int st, lalb_ctx *ctx) {
    fprintf(stderr, "%s: %s (%d) %s\n", what, lalb_status_string(st), st,
            ctx ? lalb_last_error(ctx) : "");
    return 1;
}

static int abi_only(void) {
    /* the 12 packed bytes of scales 1..8 and mins 9..16 (6-bit each) */
    static const uint8_t packed[12] = {1, 2, 3, 4, 9, 10, 11, 0x4C, 0xD5, 0xE6, 0xF7, 0x08};
    uint8_t out[16];
    lalb_ctx *ctx = NULL;
    int i, st;
    if (lalb_abi_version() != LALB_ABI_VERSION) return fail("abi version", -1, NULL);
    st = lalb_unpack_scales_6bit(packed, out);
    if (st != LALB_OK) return fail("unpack_scales_6bit", st, NULL);
    for (i = 0; i < 8; ++i)
        if (out[i] != i + 1 || out[8 + i] != i + 9) return fail("unpack_scales_6bit values", -1, NULL);
    if (lalb_unpack_scales_6bit(NULL, out) != LALB_ERR_INVALID) return fail("null check", -1, NULL);
    st = lalb_init(0, &ctx);
    if (st == LALB_OK) {
        lalb_destroy(ctx);
        printf("abi ok, device 0 is sm_100\n");
    } else if (st == LALB_ERR_DEVICE) {
        printf("abi ok, no sm_100 device\n");
    } else {
        return fail("lalb_init", st, NULL);
    }
    return 0;
}

static void *read_all(const char *path, size_t *n) {
    FILE *f = fopen(path, "rb");
    void *buf;
    long len;
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    len = ftell(f);
    fseek(f, 0, SEEK_SET);
    buf = malloc((size_t)len);
    if (buf && fread(buf, 1, (size_t)len, f) != (size_t)len) {
        free(buf);
        buf = NULL;
    }
    fclose(f);
    *n = (size_t)len;
    return buf;
}

int main(int argc, char **argv) {
    unsigned char *in, *p;
    size_t n_in = 0, wbytes;
    int32_t hdr[4];
    int rows, K, hrows, hK, st, rc = 1;
    lalb_ctx *ctx = NULL;
    void *dW = NULL, *dx = NULL, *dy = NULL, *dH = NULL, *dsw = NULL, *dxh = NULL, *dlog = NULL,
         *dam = NULL;
    float *y = NULL, *logits = NULL;
    int32_t am = -2;
    FILE *out;

    if (argc == 2 && strcmp(argv[1], "--abi-only") == 0) return abi_only();
    if (argc != 3) {
        fprintf(stderr, "usage: %s --abi-only | <in.bin> <out.bin>\n", argv[0]);
        return 2;
    }
    in = (unsigned char *)read_all(argv[1], &n_in);
    if (!in || n_in < sizeof(hdr)) return fail("read input", -1, NULL);
    memcpy(hdr, in, sizeof(hdr));
    rows = hdr[0];
    K = hdr[1];
    hrows = hdr[2];
    hK = hdr[3];
    wbytes = (size_t)rows * (size_t)(K / 256) * 144u;
    if (n_in != sizeof(hdr) + wbytes + 4u * (size_t)K + (size_t)hrows * (size_t)hK +
                    4u * (size_t)hrows + 4u * (size_t)hK)
        return fail("input size", -1, NULL);
    p = in + sizeof(hdr);

    st = lalb_init(0, &ctx);
    if (st != LALB_OK) return fail("lalb_init", st, NULL);
    if (cudaMalloc(&dW, wbytes) != cudaSuccess || cudaMalloc(&dx, 4u * (size_t)K) != cudaSuccess ||
        cudaMalloc(&dy, 4u * (size_t)rows) != cudaSuccess ||
        cudaMalloc(&dH, (size_t)hrows * (size_t)hK) != cudaSuccess ||
        cudaMalloc(&dsw, 4u * (size_t)hrows) != cudaSuccess ||
        cudaMalloc(&dxh, 4u * (size_t)hK) != cudaSuccess ||
        cudaMalloc(&dlog, 4u * (size_t)hrows) != cudaSuccess || cudaMalloc(&dam, 4) != cudaSuccess) {
        fail("cudaMalloc", -3, ctx);
        goto done;
    }
    cudaMemcpy(dW, p, wbytes, cudaMemcpyHostToDevice);
    p += wbytes;
    cudaMemcpy(dx, p, 4u * (size_t)K, cudaMemcpyHostToDevice);
    p += 4u * (size_t)K;
    cudaMemcpy(dH, p, (size_t)hrows * (size_t)hK, cudaMemcpyHostToDevice);
    p += (size_t)hrows * (size_t)hK;
    cudaMemcpy(dsw, p, 4u * (size_t)hrows, cudaMemcpyHostToDevice);
    p += 4u * (size_t)hrows;
    cudaMemcpy(dxh, p, 4u * (size_t)hK, cudaMemcpyHostToDevice);

    /* the two calls the engine's forward pass makes per token */
    st = lalb_matmul_q4_k(ctx, dW, rows, K, (const float *)dx, (float *)dy, NULL);
    if (st != LALB_OK) {
        fail("lalb_matmul_q4_k", st, ctx);
        goto done;
    }
    st = lalb_lm_head_int8_range(ctx, (const int8_t *)dH, (const float *)dsw, hK, 0, hrows,
                                 (const float *)dxh, (float *)dlog, (int32_t *)dam, NULL);
    if (st != LALB_OK) {
        fail("lalb_lm_head_int8_range", st, ctx);
        goto done;
    }
    st = lalb_device_status(ctx, 0);   /* synchronises; 0 = no bounded wait expired */
    if (st != 0) {
        fail("device status", st, ctx);
        goto done;
    }
    y = (float *)malloc(4u * (size_t)rows);
    logits = (float *)malloc(4u * (size_t)hrows);
    if (!y || !logits || cudaMemcpy(y, dy, 4u * (size_t)rows, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(logits, dlog, 4u * (size_t)hrows, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(&am, dam, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        fail("copy back", -2, ctx);
        goto done;
    }
    out = fopen(argv[2], "wb");
    if (!out) {
        fail("open output", -1, ctx);
        goto done;
    }
    fwrite(y, 4, (size_t)rows, out);
    fwrite(logits, 4, (size_t)hrows, out);
    fwrite(&am, 4, 1, out);
    fclose(out);
    rc = 0;
done:
    cudaFree(dW);
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(dH);
    cudaFree(dsw);
    cudaFree(dxh);
    cudaFree(dlog);
    cudaFree(dam);
    free(y);
    free(logits);
    free(in);
    if (ctx) lalb_destroy(ctx);
    return rc;
}
