/* CPU oracle for the AlphaZero network-evaluation hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library restates, in plain C, the
 * reference's CPU inference forward (robominds/alphazero-go,
 * src/network.cpp:228-309 in inference mode) together with everything
 * needed to build the same network and the same inputs from a seed:
 *   - the xoshiro256** / splitmix64 generator (src/rng.cpp:19-86),
 *   - Network(cfg, seed) He-normal initialisation (src/network.cpp:77-111,
 *     src/layers.cpp:14-17,29,164-167),
 *   - ParamLayout::of (src/param_layout.cpp:18-29),
 *   - the batch-norm randomisers used by the tests and the benchmark.
 * Only tests/, the smoke check and bench.py's CPU-baseline leg may load it;
 * the GPU engine never links or calls it.
 *
 * Parity pin: az_forward_f32 follows the reference's `naive` backend
 * summation order exactly (src/backend.cpp:115-140: each output element is
 * a left-to-right float sum over k of separately rounded products), so it is
 * bit-identical to the reference's own naive build; tests/golden holds the
 * fixtures made by that build (oracle/_ref) that check it.
 */
#ifndef AZ_ORACLE_H
#define AZ_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* NetConfig (include/azgo/network.hpp:23-36). planes = 2*history+2. */
typedef struct az_netcfg {
    int board;        /* n, 5..19 */
    int history;      /* H >= 1 */
    int blocks;       /* residual blocks >= 0 */
    int filters;      /* F */
    int value_hidden; /* V */
    int ownership;    /* 0/1: the ownership head */
} az_netcfg;

/* Random number generation (src/rng.cpp). */
typedef struct az_rng { uint64_t s[4]; } az_rng;
uint64_t az_splitmix64(uint64_t* x);
uint64_t az_derive_seed(uint64_t a, uint64_t b, uint64_t c, uint64_t d);
void az_rng_seed(az_rng* r, uint64_t seed);
uint64_t az_rng_next(az_rng* r);
double az_rng_uniform(az_rng* r);
int az_rng_below(az_rng* r, int n);
double az_rng_normal(az_rng* r);

/* ParamLayout (src/param_layout.cpp:18-29): which = 0 params, 1 buffers.
 * Entry names follow Network::params()/buffers() (src/network.cpp:113-165). */
int az_layout_count(const az_netcfg* cfg, int which);
int az_layout_entry(const az_netcfg* cfg, int which, int index, char* name, size_t name_cap,
                    size_t* size, size_t* offset, int* decay);
size_t az_layout_floats(const az_netcfg* cfg, int which);

/* Network(cfg, seed): He-normal conv/linear weights, zero biases, BN at
 * gamma 1, beta 0, mean 0, var 1. The arenas are zeroed first. */
void az_network_init(const az_netcfg* cfg, uint64_t seed, float* params, float* buffers);

/* Batch-norm statistics and biases that are not the identity.
 * kind 0 ("bench"): from Rng(deriveSeed(seed, 1)) in params() then
 *   buffers() order: gamma ~ U(0.5,1.5), beta ~ N(0,0.1), runMean ~ N(0,0.1),
 *   runVar ~ U(0.5,1.5); linear biases stay 0.
 * kind 1 ("test"): the reference test suite's randomNetwork
 *   (tests/test_cuda.cpp:188-204): Rng(seed + 17), gamma 0.5 + U, beta and
 *   biases 0.4U - 0.2, runVar 0.5 + U, runMean 0.4U - 0.2. */
void az_randomize(const az_netcfg* cfg, int kind, uint64_t seed, float* params, float* buffers);

/* Inputs [B][planes][area].
 * az_inputs_positions: sample b (global index first + b) draws from
 *   Rng(deriveSeed(seed, 2, first + b)): side to move = below(2) (0 black),
 *   then per point: occupied if uniform() < 0.4, colour below(2) (0 black).
 *   Encoded as encodePlanes does with one history position
 *   (src/encode.cpp:14-43): own, opponent, then the two side-to-move planes.
 * az_inputs_planes: every float below(2) from Rng(seed) (tests/test_cuda.cpp:207-211). */
void az_inputs_positions(const az_netcfg* cfg, uint64_t seed, long first, int B, float* out);
void az_inputs_planes(uint64_t seed, size_t count, float* out);

/* Network::infer in float with the naive backend's summation order.
 * logits [B][area+1], values [B], ownership [B][area] or NULL.
 * threads > 1 splits output channels over threads (bits unchanged). */
void az_forward_f32(const az_netcfg* cfg, const float* params, const float* buffers,
                    const float* input, int B, float* logits, float* values, float* ownership,
                    int threads);

/* The same network in double precision (tests/test_cuda.cpp:659-752). */
void az_forward_f64(const az_netcfg* cfg, const float* params, const float* buffers,
                    const float* input, int B, float* logits, float* values, float* ownership,
                    int threads);

#ifdef __cplusplus
}
#endif
#endif
