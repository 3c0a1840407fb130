// ref_shim.cpp - TEST INFRASTRUCTURE ONLY (never linked into the product).
//
// Compiles the reference's own CPU code for the decode hot path, unmodified,
// by #include from the reference source tree (-I <reference>/src), and
// exports it through a flat C ABI so the tests can call it with ctypes:
//
//   sampler.hpp:33-157      smoe::sample_token   (rep-penalty, temperature,
//                                                 top-k heap, top-p, draw)
//   scout/scout.cpp:77-123  smoe::scout::top_k   (softmax + partial selection
//                                                 sort + optional renorm)
//   common.hpp:294-306      smoe::matvec_bf16    (scalar path: x86 has no NEON)
//   common.hpp:245-256      smoe::rms_norm_bf16
//
// The only addition is the routing glue of decode.cpp:280-303 (gate matvec ->
// top_k(norm=false) -> renormalise over the k chosen in rank order), written
// here as a few lines of our own that call the reference functions above.
//
// Built by oracle/Makefile into oracle/_ref/libsmoe_ref.so (git-ignored).
// Flags: -O3 -ffp-contract=off (x86 g++ has no FMA contraction without
// -mfma anyway; stated so the sequential fp32 sums are plain mul+add).

#include "sampler.hpp"
#include "common.hpp"
#include "scout/scout.cpp"   // top_k() is file-static: reachable only by inclusion

#include <sstream>
#include <cstdint>
#include <cstring>

// scout.cpp registers its mmap with the Metal bridge; there is no Metal here.
extern "C" void smoe_metal_register_buffer(SmoeMetalCtx*, const void*, size_t) {}

namespace {

// Inverse of y = x ^ ((x << s) & m)
uint32_t undo_shl(uint32_t y, int s, uint32_t m) {
    uint32_t x = y;
    for (int i = 0; i < 32 / s + 1; ++i) x = y ^ ((x << s) & m);
    return x;
}
// Inverse of y = x ^ (x >> s)
uint32_t undo_shr(uint32_t y, int s) {
    uint32_t x = y;
    for (int i = 0; i < 32 / s + 1; ++i) x = y ^ (x >> s);
    return x;
}
// Inverse of the MT19937 output tempering (published constants of the
// Mersenne Twister, Matsumoto & Nishimura 1998).
uint32_t mt_untemper(uint32_t y) {
    y = undo_shr(y, 18);
    y = undo_shl(y, 15, 0xefc60000u);
    y = undo_shl(y, 7, 0x9d2c5680u);
    y = undo_shr(y, 11);
    return y;
}

// An std::mt19937 whose NEXT output is exactly `word`: the state array is
// set through the standard stream format (624 words + position), with the
// untempered word at the last slot and the position pointing at it.
std::mt19937 rng_yielding(uint32_t word) {
    std::ostringstream os;
    for (int i = 0; i < 623; ++i) os << 0u << ' ';
    os << mt_untemper(word) << ' ' << 623;
    std::istringstream is(os.str());
    std::mt19937 rng;
    is >> rng;
    return rng;
}

}  // namespace

extern "C" {

// One mt19937 output after state injection (self-check of the trick above).
uint32_t ref_mt_next_after_inject(uint32_t word) {
    std::mt19937 rng = rng_yielding(word);
    return static_cast<uint32_t>(rng());
}

// generate_canonical<float,24> applied to a generator whose next word is `word`.
float ref_canonical_from_word(uint32_t word) {
    std::mt19937 rng = rng_yielding(word);
    return std::generate_canonical<float, 24>(rng);
}

// First n outputs of std::mt19937(seed) (the engine seeds 1337, main.cpp:316).
void ref_mt19937_words(uint32_t seed, uint32_t n, uint32_t* out) {
    std::mt19937 rng(seed);
    for (uint32_t i = 0; i < n; ++i) out[i] = static_cast<uint32_t>(rng());
}

// smoe::sample_token with a caller-chosen 32-bit draw. `scores` is mutated
// in place exactly as the reference does (repetition penalty).
// scratch_k: size of the top-K candidate heap (main.cpp:324 uses
// max(top_k, 1024)); 0 selects that default.
uint32_t ref_sample_token(float* scores, uint32_t vocab, float temperature,
                          float top_p, uint32_t top_k, float rep_penalty,
                          const uint32_t* history, uint32_t history_len,
                          uint32_t word, uint32_t scratch_k) {
    smoe::SamplerConfig cfg{vocab, temperature, top_p, top_k, rep_penalty};
    if (scratch_k == 0) scratch_k = std::max(top_k, 1024u);
    smoe::SamplerScratch scratch(scratch_k, vocab);
    std::mt19937 rng = rng_yielding(word);
    return smoe::sample_token(scores, cfg, history, history_len, rng, scratch);
}

uint32_t ref_top_k(const float* scores, uint32_t n, uint32_t k,
                   uint32_t* out_idx, float* out_w, int norm) {
    return smoe::scout::top_k(scores, n, k, out_idx, out_w, norm != 0);
}

void ref_matvec_bf16(float* out, const uint16_t* w, const float* in,
                     uint32_t rows, uint32_t cols) {
    smoe::matvec_bf16(out, w, in, rows, cols);
}

void ref_rms_norm_bf16(float* x, const uint16_t* w, uint32_t n) {
    smoe::rms_norm_bf16(x, w, n);
}

// decode.cpp:280-303: gate matvec, top-(k) with norm=false, then renormalise
// the k weights by their sequential sum (when norm_topk_prob).
uint32_t ref_route(const float* x, const uint16_t* gate_w, uint32_t n_experts,
                   uint32_t d_model, uint32_t k, int norm_topk_prob,
                   float* logits_out, uint32_t* ids, float* weights) {
    smoe::matvec_bf16(logits_out, gate_w, x, n_experts, d_model);
    uint32_t nsel = smoe::scout::top_k(logits_out, n_experts, k, ids, weights, false);
    float w_sum = 0.0f;
    for (uint32_t e = 0; e < nsel; ++e) w_sum += weights[e];
    const float w_inv = (norm_topk_prob && w_sum > 0.0f) ? 1.0f / w_sum : 1.0f;
    for (uint32_t e = 0; e < nsel; ++e) weights[e] = weights[e] * w_inv;
    return nsel;
}

}  // extern "C"
