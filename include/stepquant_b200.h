/*
 * stepquant_b200 -- C ABI of the B200 (sm_100a) packed-state recurrent decode path.
 *
 * The reference (STEPQuant) is Python calling Triton/Gluon kernels; it has no
 * C/FFI layer of its own.  Each entry point below replaces one reference
 * operation on this path and names it (file:line inside the reference tree).
 * The Python mirror in ``stepquant_b200`` binds these with ctypes; a C or C++
 * host binds them directly.
 *
 * Conventions
 *  - All tensor pointers are device pointers unless a parameter says "host".
 *    Buffers are owned by the caller; no entry point allocates device memory.
 *  - ``stream`` is a cudaStream_t (0 = legacy default stream).  Each device
 *    entry point that replaces a reference operation (all but
 *    sq_step_async_noalloc) only enqueues work: it never synchronizes, never
 *    reads device memory on the host and is therefore legal inside CUDA-graph
 *    capture.
 *  - Return value: SQ_OK or an SQ_ERR_* code for argument errors detected on
 *    the host before launch (the reference raises ValueError at the same
 *    points), or SQ_ERR_CUDA when the launch itself failed.
 *  - ``status`` (optional, may be NULL) is a device int32 word.  Kernels OR
 *    SQ_STATUS_* bits into it for conditions only visible on the device
 *    (a slot index outside the pool).  Such requests are skipped: zero output,
 *    no page write.
 *  - A slot index <= 0 marks a padded request (the reference's sentinel slot
 *    0): its output row is zero and its page is neither read nor written.
 */
#ifndef STEPQUANT_B200_H
#define STEPQUANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *sq_stream_t; /* == cudaStream_t */

enum sq_error {
    SQ_OK = 0,
    SQ_ERR_ARGUMENT = 1,    /* null pointer, negative size, bad enum          */
    SQ_ERR_SHAPE = 2,       /* shape / stride / divisibility violated          */
    SQ_ERR_UNSUPPORTED = 3, /* valid for the reference but not built here      */
    SQ_ERR_CUDA = 4,        /* kernel launch or CUDA runtime failure           */
    SQ_ERR_CAPACITY = 5     /* batch larger than the caller's scratch capacity */
};

enum sq_status_bits {
    SQ_STATUS_SLOT_RANGE = 1, /* a slot index >= num_slots was skipped */
    SQ_STATUS_TIMEOUT = 2     /* a bounded device wait gave up (results incomplete) */
};

enum sq_dtype { SQ_F32 = 0, SQ_BF16 = 1, SQ_F16 = 2 };
enum sq_architecture { SQ_GDN = 0, SQ_KDA = 1 };

/*
 * One layer's quantization plan and page layout (QuantizationPlan,
 * stepquant/quantization.py:7-26, plus the tables PackedStatePool builds in
 * stepquant/kernels/pool.py:85-91).  Device tables:
 *   bits     [heads*keys]        2, 4, 6, 8 or 16 (16 = fp16 pivot row)
 *   impact   [heads*keys]        row weights w > 0
 *   offsets  [heads*keys+heads]  code/pivot byte offset of each key row, then
 *                                each head's byte stride between value tiles
 *   rows     [heads*keys]        byte offset of each row's fp16 scale(s), -1 = pivot
 *   columns  [heads]             byte offset of each head's fp16 column scales, -1 = none
 *   bits_host [heads*keys]       optional HOST copy of bits (may be NULL); when
 *                                given, the host skips launches that no head needs
 * The tables must be those sq_packed_layout produces for `bits`.
 * Supported shapes: keys, values in {4,...,128} (powers of two); GDN needs
 * values % value_group_size == 0 and at most 32 value groups.
 */
typedef struct sq_plan {
    int32_t architecture; /* SQ_GDN or SQ_KDA */
    int32_t heads;
    int32_t keys;
    int32_t values;
    int32_t value_group_size;
    int32_t storage;      /* pages: 0 packed codes (tiles of 16 / 4 values), 1 byte carriers;
                             baseline formats: 2 symmetric groups (sym_int*), 3 dual axis (dsq_int*) */
    int64_t page_bytes;
    const int32_t *bits;
    const float *impact;
    const int32_t *offsets;
    const int32_t *rows;
    const int32_t *columns;
    const int32_t *bits_host;
} sq_plan;

/*
 * Inputs of one decode step (PackedStatePool.step arguments,
 * stepquant/kernels/pool.py:200-215).
 *   q, k  [batch, qk_heads, keys] with request stride q_stride / k_stride
 *         (elements); head vectors contiguous.  Value head h reads qk head
 *         h / (heads / qk_heads).
 *   v     [batch, heads*values] with request stride v_stride.
 *   g     GDN [batch, heads], KDA [batch, heads, keys], contiguous: the log
 *         decay, or the raw gate input when a_log != NULL.
 *   beta  [batch, heads] contiguous: beta, or its logit when a_log != NULL.
 *   a_log [heads] and dt_bias ([heads] GDN / [heads*keys] KDA), fp32, or NULL.
 *   out   [batch, heads, values] in io_dtype.
 * With a_log: log decay = -exp(a_log) * softplus(g + dt_bias) and
 * beta = sigmoid(beta) (fused.py:170-174).  With normalize: q and k are L2
 * normalised with eps 1e-6; q is then multiplied by scale.
 */
typedef struct sq_step_args {
    const void *q;
    const void *k;
    const void *v;
    int64_t q_stride;
    int64_t k_stride;
    int64_t v_stride;
    int32_t qk_heads;
    int32_t io_dtype; /* dtype of q, k, v and out */
    const void *g;
    const void *beta;
    int32_t gate_dtype; /* dtype of g and beta */
    int32_t normalize;
    const float *a_log;
    const float *dt_bias;
    float scale;
    int32_t reserved;
    void *out;
} sq_step_args;

/* Library version (major * 10000 + minor * 100 + patch). */
int32_t sq_version(void);

/* Human-readable text for an sq_error code. */
const char *sq_error_string(int32_t code);

/*
 * Host: page layout tables of a plan (stepquant/kernels/pool.py:19-66,
 * ``packed_layout``).  bits_host is [heads*keys] host memory; the outputs are
 * host arrays of heads*keys+heads, heads*keys and heads entries.  storage: 0 =
 * packed, 1 = byte carriers (one int8 level per value; every device entry point accepts both).
 */
int32_t sq_packed_layout(int32_t architecture, int32_t heads, int32_t keys, int32_t values,
                         int32_t value_group_size, const int32_t *bits_host, int32_t storage,
                         int32_t *offsets_out, int32_t *rows_out, int32_t *columns_out,
                         int64_t *page_bytes_out);

/*
 * Dense fp32 state [batch, heads, keys, values] -> pages[slots[i]]
 * (PackedStatePool.encode / _writeback, stepquant/kernels/pool.py:184-190,319-331;
 * quantizer = fit_state, stepquant/quantization.py:54-98).  Only code bytes,
 * pivots and scales are written; alignment padding keeps its contents.
 */
int32_t sq_encode(const sq_plan *plan, const float *state, const int64_t *slots, int32_t batch,
                  uint8_t *pages, int64_t num_slots, int32_t *status, sq_stream_t stream);

/*
 * pages[slots[i]] -> dense fp32 [batch, heads, keys, values]
 * (PackedStatePool.decode, stepquant/kernels/pool.py:192-198; fused.py:19-59).
 */
int32_t sq_decode(const sq_plan *plan, const uint8_t *pages, int64_t num_slots, const int64_t *slots,
                  int32_t batch, float *state, int32_t *status, sq_stream_t stream);

/*
 * One synchronous decode step, fused: unpack, gated delta rule, readout,
 * requantize (fit_state), repack, in place on pages[slots[i]]
 * (PackedStatePool.step without a writeback stream, stepquant/kernels/pool.py:200-282,
 * whose math is core.delta_step + fit_state).  state_out (optional,
 * [batch, heads, keys, values] fp32) receives the updated state before
 * requantization.
 */
int32_t sq_step(const sq_plan *plan, uint8_t *pages, int64_t num_slots, const int64_t *slots,
                int32_t batch, const sq_step_args *args, float *state_out, int32_t *status,
                sq_stream_t stream);

/* Floats of per-request scratch that sq_readout writes and sq_writeback reads. */
int64_t sq_scratch_floats(const sq_plan *plan);

/*
 * Foreground half of an asynchronous step (readout.py:8-121 / segment_read.py
 * launched from pool.py:239-258): unpack, gated delta rule and readout.  Writes
 * out, fp16 pivot rows in place, per-request scratch
 * ([batch, sq_scratch_floats] fp32) and stable_slots[i] = slots[i].
 */
int32_t sq_readout(const sq_plan *plan, uint8_t *pages, int64_t num_slots, const int64_t *slots,
                   int32_t batch, const sq_step_args *args, float *scratch, int64_t *stable_slots,
                   int32_t *status, sq_stream_t stream);

/*
 * Background half (PackedStatePool._finish_update, pool.py:299-316: rows.py +
 * fit.py): rebuilds the updated state from the page and the scratch of
 * sq_readout, requantizes and repacks the integer rows of
 * pages[stable_slots[i]].  Produces the same bytes as sq_step.  state_out is
 * reserved and must be NULL (sq_step's state_out exposes the pre-quantization
 * state).
 */
int32_t sq_writeback(const sq_plan *plan, uint8_t *pages, int64_t num_slots,
                     const int64_t *stable_slots, int32_t batch, const float *scratch,
                     float *state_out, int32_t *status, sq_stream_t stream);

/*
 * fit_state on the device (stepquant/quantization.py:54-98).
 *   x      [batch, heads, keys, values] fp32
 *   z      [batch, heads, keys, values] int16 integer levels (all rows)
 *   r      [batch, heads, keys] fp16 bits (uint16) row scales (all rows)
 *   c      [batch, heads, values] fp16 bits column scales
 *   r2     [batch, two-bit GDN heads, keys, values/value_group_size] fp16 bits, or NULL
 *   recon  [batch, heads, keys, values] fp32 reconstruction, or NULL
 */
int32_t sq_fit_state(const sq_plan *plan, const float *x, int32_t batch, int16_t *z, uint16_t *r,
                     uint16_t *c, uint16_t *r2, float *recon, sq_stream_t stream);

/*
 * No counterpart in the reference.  The asynchronous decode step (sq_readout
 * then sq_writeback on `stream`) for callers that cannot allocate device memory
 * when they step, e.g. a server that reserves its whole device budget at
 * start-up, or a binding with no device allocator of its own.  Its scratch is
 * a 16 MiB file-scope device array of the library (sq_noalloc_scratch_bytes())
 * instead of caller buffers; a call needs round_up(batch*8, 256) +
 * batch * sq_scratch_floats(plan) * 4 bytes of it and returns SQ_ERR_CAPACITY
 * above that.  All calls share the array, so calls that overlap on the GPU
 * race.  The first call on a device looks up the array's address; make it
 * before any stream capture.  Writes the same out and page bytes as
 * sq_readout + sq_writeback.
 */
int32_t sq_step_async_noalloc(const sq_plan *plan, uint8_t *pages, int64_t num_slots, const int64_t *slots,
                              int32_t batch, const sq_step_args *args, int32_t *status, sq_stream_t stream);

/* Size in bytes of the file-scope scratch array used by sq_step_async_noalloc. */
int64_t sq_noalloc_scratch_bytes(void);

/*
 * Writeback stream with an SM budget (replaces the green-context stream that
 * stepquant/kernels/resources.py:19-53 builds through the CUDA driver from
 * Python).  A non-blocking stream of a green context that owns at least
 * `sm_budget` SMs of `device` (the driver rounds up to its SM-group size);
 * kernels launched on it run on those SMs only.  One context and stream per
 * (device, budget), created on the first call and kept until the process
 * exits.  Out (host): *stream, *actual_sms (SMs granted), *total_sms (the
 * device's SMs, also set when the budget is rejected).  SQ_ERR_ARGUMENT for a
 * budget outside 1..total_sms or a bad device; SQ_ERR_UNSUPPORTED when the
 * driver has no green contexts; SQ_ERR_CUDA when the driver refuses.
 */
int32_t sq_budget_stream(int32_t device, int32_t sm_budget, sq_stream_t *stream, int32_t *actual_sms,
                         int32_t *total_sms);

/* packing.pack (stepquant/packing.py:6-14): codes int16 [n] -> little-endian bytes. */
int32_t sq_pack(const int16_t *codes, int64_t n, int32_t bits, uint8_t *out, sq_stream_t stream);

/* Bytes sq_pack writes for n codes. */
int64_t sq_packed_bytes(int64_t n, int32_t bits);

/* packing.unpack (stepquant/packing.py:17-22): bytes -> int16 codes [count]. */
int32_t sq_unpack(const uint8_t *data, int64_t count, int32_t bits, int16_t *out, sq_stream_t stream);

/*
 * FP32 state pool decode step, the reference's FP32 baseline
 * (stepquant/kernels/floating.py:20-53): state [num_slots, heads, keys, values]
 * fp32 updated in place for slots[i] > 0.
 */
int32_t sq_fp32_step(float *state, int64_t num_slots, int32_t heads, int32_t keys, int32_t values,
                     int32_t kda, const int64_t *slots, int32_t batch, const sq_step_args *args,
                     int32_t *status, sq_stream_t stream);

/*
 * GDN chunked prefill: the state pass that produces each sequence's state
 * after its prompt.  It replaces the SGLang chunk kernel
 * (TritonGDNKernel.extend) that stepquant/sglang/runtime.py:193-202 calls
 * between PackedStatePool.decode and PackedStatePool.encode; the recurrence
 * is core.delta_step (stepquant/core.py:5-15) applied token by token.
 * Tokens of num_seqs sequences are concatenated: sequence n owns tokens
 * [cu_seqlens[n], cu_seqlens[n+1]), clamped to [0, tokens).
 *   q, k   [tokens, qk_heads, keys] bf16, token rows q_stride / k_stride
 *          elements apart (16-byte aligned rows)
 *   v      [tokens, heads, values] bf16, rows v_stride apart
 *   g      [tokens, heads] fp32 log decay; beta [tokens, heads] fp32
 *   initial_state [num_seqs, heads, keys, values] fp32, or NULL for zeros
 *   final_state   [num_seqs, heads, keys, values] fp32 (may equal initial_state)
 *   out    [tokens, heads, values] bf16: o_t = q_t^T S_t
 * normalize: q and k are L2 normalised per token (eps 1e-6), q is then
 * multiplied by scale.  Value head h reads qk head h / (heads / qk_heads).
 *   workspace  caller-owned device buffer of at least
 *          sq_gdn_prefill_workspace_bytes(tokens, num_seqs, heads) bytes,
 *          256-byte aligned (per-chunk intermediates; SQ_ERR_CAPACITY if short)
 * The pass runs in 64-token chunks in the WY/UT form on tensor cores (bf16
 * operands, fp32 accumulation; the state is carried in fp32): one kernel
 * prepares every chunk in parallel, a second walks each sequence's chunks.
 * keys = values = 128 only (SQ_ERR_UNSUPPORTED otherwise).
 */
typedef struct sq_prefill_args {
    const void *q;
    const void *k;
    const void *v;
    int64_t q_stride;
    int64_t k_stride;
    int64_t v_stride;
    int32_t io_dtype; /* SQ_BF16 */
    int32_t qk_heads;
    int32_t heads;
    int32_t keys;
    int32_t values;
    int32_t normalize;
    float scale;
    int32_t num_seqs;
    int32_t tokens;
    const int32_t *cu_seqlens;
    const float *g;
    const float *beta;
    const float *initial_state;
    float *final_state;
    void *out;
    void *workspace;
    int64_t workspace_bytes;
    int32_t *status; /* device int32 for SQ_STATUS_* bits, or NULL */
} sq_prefill_args;

int64_t sq_gdn_prefill_workspace_bytes(int32_t tokens, int32_t num_seqs, int32_t heads);
int32_t sq_gdn_prefill(const sq_prefill_args *args, sq_stream_t stream);

/*
 * KDA prefill: the same state pass for layers with a per-key-channel decay
 * (Kimi-Delta-Attention).  It replaces the SGLang KDA chunk kernel that the
 * same hook (stepquant/sglang/runtime.py:193-202) calls; the recurrence is
 * core.delta_step (stepquant/core.py:5-15) with log_decay [heads, keys].
 * Arguments as for sq_gdn_prefill except
 *   g      [tokens, heads, keys] fp32 log decay per key channel, 16-byte
 *          aligned base
 *   initial_state, final_state: 16-byte aligned
 *   workspace, workspace_bytes, status: unused (may be NULL / 0)
 * The pass keeps each (sequence, head) state in fp32 registers and walks the
 * tokens in order (fp32 arithmetic throughout); keys = values = 128 only.
 */
int32_t sq_kda_prefill(const sq_prefill_args *args, sq_stream_t stream);

/*
 * Self-test of the division used by the register-resident decode kernels: for
 * i < n, out[i] = a[i] / b[i] computed with a correctly rounded reciprocal of
 * the fp16 value b[i] (given as its bits) and one Markstein correction.  It
 * must equal IEEE round-to-nearest a[i] / b[i] whenever the quotient is a
 * normal number; tests compare it with the device's IEEE division.
 */
int32_t sq_selftest_fp16_division(const float *a, const uint16_t *b, float *out, int64_t n, sq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* STEPQUANT_B200_H */
