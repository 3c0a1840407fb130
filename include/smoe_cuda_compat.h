/*
 * smoe_cuda_compat.h - name shim for the reference engine.
 *
 * Lets src/decode.cpp, src/prefill.cpp, src/main.cpp and src/scout/scout.cpp
 * of the reference compile unchanged against libsmoe_cuda: include this in
 * place of compute/metal_bridge.h. Every smoe_metal_X of metal_bridge.h
 * (:47-224) maps to the smoe_cuda_X of smoe_cuda.h with the same arguments.
 * Weight pointers handed to the FFN entries must be device pointers into the
 * resident expert arena.
 */
#pragma once
#include "smoe_cuda.h"

typedef SmoeCudaCtx SmoeMetalCtx;
#define smoe_metal_init                     smoe_cuda_init
#define smoe_metal_destroy                  smoe_cuda_destroy
#define smoe_metal_fused_ffn                smoe_cuda_fused_ffn
#define smoe_metal_wait                     smoe_cuda_wait
#define smoe_metal_fused_ffn_group          smoe_cuda_fused_ffn_group
#define smoe_metal_fused_ffn_batch          smoe_cuda_fused_ffn_batch
#define smoe_metal_wait_ffn_batch           smoe_cuda_wait_ffn_batch
#define smoe_metal_scout_matvec_bf16        smoe_cuda_scout_matvec_bf16
#define smoe_metal_register_buffer          smoe_cuda_register_buffer
#define smoe_metal_kernel_dispatches        smoe_cuda_kernel_dispatches
