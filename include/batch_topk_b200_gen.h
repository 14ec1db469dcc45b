/*
 * batch_topk_b200_gen.h -- device-side generation of the benchmark inputs (no reference
 * counterpart; the reference's own test and benchmark fill their inputs on the host).
 *
 * Each call fills d_out[0 .. n) with fp16 bit patterns for flat element indices
 * idx0 .. idx0 + n - 1 of one (seed, stream) sequence, bit-identical to the host generators
 * of batch_topk_b200/workloads.py, so a shard of any configuration can be generated in place
 * on its own device.  Asynchronous on `stream`; returns a cudaError_t code.
 */
#ifndef BATCH_TOPK_B200_GEN_H_
#define BATCH_TOPK_B200_GEN_H_

#ifdef __cplusplus
extern "C" {
#endif

/* N(0, sigma^2) by Box-Muller from counters 2i and 2i+1, rounded to fp16. */
int bt_gen_normal(void* d_out, long long n, unsigned long long idx0, unsigned long long seed,
                  unsigned long long stream_id, double sigma, void* stream);

/* lo + (hi - lo) * U[0, 1), rounded to fp16. */
int bt_gen_uniform(void* d_out, long long n, unsigned long long idx0, unsigned long long seed,
                   unsigned long long stream_id, double lo, double hi, void* stream);

/* d_levels256[top byte of the counter draw]: a uniform pick from a 256-entry fp16 table. */
int bt_gen_levels(void* d_out, long long n, unsigned long long idx0, unsigned long long seed,
                  unsigned long long stream_id, const void* d_levels256, void* stream);

/* In place: entries whose uniform draw is below p become fill_bits. */
int bt_gen_mask(void* d_inout, long long n, unsigned long long idx0, unsigned long long seed,
                unsigned long long stream_id, double p, unsigned short fill_bits, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BATCH_TOPK_B200_GEN_H_ */
