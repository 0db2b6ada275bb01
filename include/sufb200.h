/*
 * sufb200.h -- C ABI of the B200-native PFSS evaluation engine (libsufb200.so).
 *
 * Plain pointers and sizes only.  "d_" arguments are device pointers on the
 * context's device; everything else is host memory.  `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  Every entry
 * point returns SUFB200_OK (0) or a negative SUFB200_ERR_* code and records a
 * message retrievable with sufb200_last_error() (thread-local).  There is no
 * CPU fallback: a missing device, a failed launch or a rejected argument is
 * an error.
 *
 * Device-side key checks (header fields of device-resident keys) are
 * reported through a per-context status word: sufb200_ctx_sync() waits for
 * the stream and returns SUFB200_ERR_KEY if any kernel flagged a bad key
 * since the last sync (the outputs of such elements are zero).
 *
 * Each comment names the reference interface (ponyyuhan/SUF, path:line)
 * that the entry point replaces.
 */
#ifndef SUFB200_H_
#define SUFB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SUFB200_OK 0
#define SUFB200_ERR_INVALID (-1)      /* bad argument (null pointer, size, range) */
#define SUFB200_ERR_CUDA (-2)         /* CUDA runtime error (launch, copy, device) */
#define SUFB200_ERR_KEY (-3)          /* key blob header / size mismatch */
#define SUFB200_ERR_UNSUPPORTED (-4)  /* valid but outside this engine's scope */
#define SUFB200_ERR_NOT_READY (-5)    /* sufb200_prg_init not called yet */
#define SUFB200_ERR_COMM (-6)         /* NCCL error or timeout in the paired-GPU open */

#define SUFB200_GROUP_ADD 0 /* myl7 u128_le group: additive shares mod 2^64 (low 8 bytes) */
#define SUFB200_GROUP_XOR 1 /* myl7 bytes group: XOR shares */

typedef struct sufb200_ctx_s* sufb200_ctx;

/* ---- library / context -------------------------------------------------- */

/* ABI version (major*10000 + minor*100 + patch). */
int sufb200_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* sufb200_last_error(void);

#define SUFB200_HOST_ONLY (-1) /* device argument of a dealer-only context */

/* Bind a context to `device` (cudaSetDevice on the calling thread), build
 * the AES tables and measure the shared-memory layout.  device =
 * SUFB200_HOST_ONLY makes a dealer-only context (no GPU needed) that accepts
 * sufb200_prg_init and the keygen calls; its evaluation calls return
 * SUFB200_ERR_UNSUPPORTED.  One context per
 * party per device, like one GpuPfssBackend per party
 * (src/demo/bench_suf_transformer.cpp:902-903); calls on one context must be
 * serialised by the caller (the reference guards its backend with a mutex,
 * cuda/pfss_backend_gpu.cu:529). */
int sufb200_ctx_create(int device, sufb200_ctx* out);
int sufb200_ctx_destroy(sufb200_ctx ctx);

/* Wait for `stream`, then report and clear the device status word. */
int sufb200_ctx_sync(sufb200_ctx ctx, void* stream);

/* Number of SMs of the context's device (grid sizing reference). */
int sufb200_ctx_sm_count(sufb200_ctx ctx);

/* Measured ceiling of the shared-memory AES-128 engine on this device: AES
 * blocks per second of the DCF walk's two-block MMO step with no other work
 * (every SM, ~1 ms; synchronises the device).  The roofline denominator of
 * the DCF kernels.  No counterpart in the reference. */
int sufb200_probe_aes_engine(sufb200_ctx ctx, double* blocks_per_s);

/* ---- myl7 PRG-tree DCF --------------------------------------------------- */

/* Install the fixed AES-128-MMO PRG keys: state[16j .. 16j+16) is key j,
 * j = 0..3 (len >= 64; the reference build passes kBlocks*16 = 128 bytes).
 * Replaces prg_init, third_party/myl7_fss/src/prg/aes128_mmo.c:16-31. */
int sufb200_prg_init(sufb200_ctx ctx, const uint8_t* state, size_t len);

/* Bytes of one party's key for `in_bits` and `payload_len`
 * (include/proto/myl7_fss_backend.hpp:156-159). */
size_t sufb200_myl7_key_bytes(int in_bits, int payload_len);

/* Dealer: one key pair for f(x) = payload if x < alpha else 0, with the
 * party seeds supplied by the caller (16 bytes per 16-byte payload chunk).
 * Byte-identical to Myl7FssBackend::gen_dcf (myl7_fss_backend.hpp:131-213,
 * which draws the seeds from std::random_device) around dcf_gen
 * (third_party/myl7_fss/src/dcf.c:42-142).  Host computation. */
int sufb200_myl7_gen(sufb200_ctx ctx, int group, int in_bits, uint64_t alpha, const uint8_t* payload,
                     int payload_len, const uint8_t* seeds0, const uint8_t* seeds1, uint8_t* key0,
                     uint8_t* key1);

/* Dealer, batched: n key pairs (alphas[i], same payload), seeds0/1 hold
 * 16*chunks bytes per element; keys0/1 are [n][key_bytes].  OpenMP. */
int sufb200_myl7_gen_batch(sufb200_ctx ctx, int group, int in_bits, const uint64_t* alphas, size_t n,
                           const uint8_t* payload, int payload_len, const uint8_t* seeds0, const uint8_t* seeds1,
                           uint8_t* keys0, uint8_t* keys1);

/* Evaluate myl7 keys (one 16-byte chunk, out_bytes <= 8) at d_xs[i], on the
 * device.  broadcast = 0: d_keys is [n][key_bytes]; broadcast = 1: one key
 * for all n.  d_out is [n][out_bytes] (little-endian low bytes of the group
 * element).  Replaces Myl7FssBackend::eval_dcf per element
 * (myl7_fss_backend.hpp:215-256) and, for this key format,
 * PfssGpuStagedEval::eval_dcf_many_u64_device[_broadcast]
 * (include/proto/backend_gpu.hpp:17-38). */
int sufb200_myl7_dcf_eval(sufb200_ctx ctx, int group, int in_bits, const uint8_t* d_keys, size_t key_bytes,
                          int broadcast, const uint64_t* d_xs, size_t n, int out_bytes, void* d_out,
                          void* stream);

/* Host-buffer form of the same evaluation: keys, xs and outs in host memory
 * (copied in and out inside the call; returns after the result is in outs).
 * Replaces PfssBackendBatch::eval_dcf_many_u64
 * (include/proto/pfss_backend_batch.hpp:11-28) for myl7 keys. */
int sufb200_myl7_dcf_eval_host(sufb200_ctx ctx, int group, int in_bits, const uint8_t* keys, size_t key_bytes,
                               int broadcast, const uint64_t* xs, size_t n, int out_bytes, uint8_t* outs);

/* ---- fused truncation / ARS bundle ------------------------------------- */

#define SUFB200_TRUNC_FAITHFUL_TR 0
#define SUFB200_TRUNC_FAITHFUL_ARS 1
#define SUFB200_TRUNC_GAPARS 2

/* One party's public bundle description.  Query q is a DCF on the low
 * q_bits[q] bits of x^ with AddU64 payload 1 (compile_suf_to_pfss_two_programs,
 * src/compiler/suf_to_pfss.cpp:300-556; composite_gen_trunc_gate,
 * include/gates/composite_fss.hpp:645-833).  Boolean outputs follow the
 * AddU64 plan of composite_eval_batch_backend (composite_fss.hpp:1385-1638):
 *   carry = [party0] - (b - a + carry_w) with a = q[carry_a], b = q[carry_b]
 *   sign  = b - a + sign_w with a = q[sign_a], b = q[sign_b]
 *   wrap  = q[wrap_q]
 * (-1 = constant 0), then the postproc hook of `kind`
 * (include/gates/postproc_hooks.hpp:173-376). */
typedef struct sufb200_trunc_desc {
  int32_t kind, frac_bits, party, nq;
  int32_t q_bits[4];
  int32_t carry_a, carry_b, sign_a, sign_b, wrap_q, reserved;
  uint64_t carry_w, sign_w; /* this party's shares of the rotation wrap bits */
  uint64_t haty;            /* base coefficient share + r_out share */
  uint64_t r_hi;            /* share of r_in >> f */
  uint64_t m;               /* GapARS: share of 2^(64-f) * MSB(r_in) */
} sufb200_trunc_desc;

/* Dealer for one bundle: draws r_in and the share splits from
 * mt19937_64(rng_seed) in the order of composite_gen_trunc_gate, fills both
 * parties' descriptors and writes the nq query thresholds to thetas[4];
 * returns r_in through *r_in_out.  The caller then makes one myl7 key pair
 * per query (in_bits = q_bits[q], alpha = thetas[q], payload = u64 1 LE). */
int sufb200_trunc_gen(int kind, int frac_bits, uint64_t rng_seed, sufb200_trunc_desc* d0, sufb200_trunc_desc* d1,
                      uint64_t* thetas, uint64_t* r_in_out);

/* Fused bundle evaluation: all nq broadcast DCFs, the boolean plan and the
 * postproc in one launch.  keys[q] (host) is this party's myl7 key of query q
 * (ADD group, 8-byte payload).  d_y is [n]; d_bools ([n][3] = carry, sign,
 * wrap shares) may be NULL.  Replaces the AddU64 truncation branch of
 * composite_eval_batch_backend followed by
 * FaithfulTruncPostProc / FaithfulArsPostProc / GapArsPostProc::run_batch. */
int sufb200_trunc_bundle_eval(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                              const size_t* key_bytes, const uint64_t* d_xhat, size_t n, uint64_t* d_y,
                              uint64_t* d_bools, void* stream);

/* One party's bundle over a bucket of jobs that share its keys (the bucket
 * step of PfssSuperBatch::flush_eval, src/runtime/pfss_superbatch.cpp:
 * 251-975, which concatenates the jobs' x^ with one device memcpy per job,
 * :801-845): job j's x^ is d_xhat[j][0..n[j]) and its result goes to
 * d_y[j].  One gather launch, one bundle evaluation over the whole bucket,
 * one scatter launch (per 48 jobs).  Host arrays of device pointers. */
int sufb200_trunc_bundle_eval_jobs(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                                   const size_t* key_bytes, const uint64_t* const* d_xhat, const size_t* n,
                                   uint64_t* const* d_y, int njobs, void* stream);

/* Both parties' bundles over the same public x^ on one GPU (desc0 / keys0 of
 * party 0, desc1 / keys1 of party 1): batches below the shared-prefix size
 * run in ONE launch with one lane per (party, element, query); larger ones
 * run sufb200_trunc_bundle_eval per party.  d_y0 / d_y1 are [n]. */
int sufb200_trunc_bundle_eval_pair(sufb200_ctx ctx, const sufb200_trunc_desc* desc0, const uint8_t* const* keys0,
                                   const size_t* key_bytes0, const sufb200_trunc_desc* desc1,
                                   const uint8_t* const* keys1, const size_t* key_bytes1, const uint64_t* d_xhat,
                                   size_t n, uint64_t* d_y0, uint64_t* d_y1, void* stream);
/* The same with every query key already in device memory (d_keys0[q],
 * d_keys1[q]: dealer material kept resident, any alignment; sizes on the
 * host): nothing is copied from the host, so a sequence of these calls can be
 * captured in a CUDA graph.  Key headers are checked on the device (status:
 * bad key header through sufb200_ctx_sync). */
int sufb200_trunc_bundle_eval_pair_dev(sufb200_ctx ctx, const sufb200_trunc_desc* desc0,
                                       const uint8_t* const* d_keys0, const size_t* key_bytes0,
                                       const sufb200_trunc_desc* desc1, const uint8_t* const* d_keys1,
                                       const size_t* key_bytes1, const uint64_t* d_xhat, size_t n, uint64_t* d_y0,
                                       uint64_t* d_y1, void* stream);

/* The same pair in two steps, for bundles whose queries are all at most 16
 * bits wide (the f-bit carries of GapARS truncations), at any batch size.
 * A party's tables hold each query's evaluations over its whole domain and
 * depend on that party's keys only, not on x^, so they can be computed on
 * another stream while x^ is still being produced, or once per key set.
 * sufb200_trunc_tables_bytes: one party's table size (0 when a query is
 * wider than 16 bits); sufb200_trunc_tables_dev fills one party's tables
 * (d_tables 256-byte aligned); sufb200_trunc_bundle_eval_pair_tables_dev
 * runs both parties' main pass over x^ against them (the same outputs as
 * sufb200_trunc_bundle_eval_pair_dev, one launch, no tree walk). */
size_t sufb200_trunc_tables_bytes(const sufb200_trunc_desc* desc);
int sufb200_trunc_tables_dev(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* d_keys,
                             const size_t* key_bytes, void* d_tables, size_t tables_bytes, void* stream);
/* Many bundles' tables (either party's) in as few launches as the keys
 * allow (16 keys per launch): descs[count], d_keys / key_bytes [count][4]
 * (the layout of the softmax / LayerNorm party structs' trunc_keys),
 * d_tables / tables_bytes [count]; a NULL d_tables[i] skips bundle i. */
int sufb200_trunc_tables_many_dev(sufb200_ctx ctx, int count, const sufb200_trunc_desc* descs,
                                  const uint8_t* const* d_keys, const size_t* key_bytes, void* const* d_tables,
                                  const size_t* tables_bytes, void* stream);
int sufb200_trunc_bundle_eval_pair_tables_dev(sufb200_ctx ctx, const sufb200_trunc_desc* desc0,
                                              const uint8_t* const* d_keys0, const size_t* key_bytes0,
                                              const void* d_tables0, const sufb200_trunc_desc* desc1,
                                              const uint8_t* const* d_keys1, const size_t* key_bytes1,
                                              const void* d_tables1, const uint64_t* d_xhat, size_t n, uint64_t* d_y0,
                                              uint64_t* d_y1, void* stream);

/* Host-buffer form: xhat, y (and bools, may be NULL) in host memory; copies
 * in and out inside the call and returns when y is on the host.  Replaces
 * composite_eval_batch_backend with a host CompositeBatchInput::hatx
 * (composite_fss.hpp:155-229) followed by the kind's postproc hook. */
int sufb200_trunc_bundle_eval_host(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                                   const size_t* key_bytes, const uint64_t* xhat, size_t n, uint64_t* y,
                                   uint64_t* bools);

/* Per-element masks (the reference's SUF_PER_ELEMENT_MASKS=1: one whole gate
 * per element, compiler::lower_truncation_gate with per_element_masks,
 * include/compiler/truncation_lowering.hpp:91-125, evaluated element by
 * element by TruncTask).  sufb200_trunc_gen_elem deals n such gates: element
 * i is sufb200_trunc_gen(kind, frac_bits, rng_seed + i * 0x9E3779B97F4A7C15);
 * shape0/1 get the fixed query slots (64-bit queries first, then the two
 * f-bit carry queries: TR [64, f, f], ARS [64, 64, f, f], GapARS [f, f]);
 * thetas[4 i + q] is element i's threshold for slot q (an element without
 * carry queries, r_low = 0, gets 0 in the f-bit slots and its plan marks the
 * carry absent); words[6 i ..] per party = carry_w, sign_w, haty, r_hi, m
 * and the plan (query indices carry_a, carry_b, sign_a, sign_b, wrap_q, 4
 * bits each, 0xF = absent); r_in[i] is element i's mask.  The caller makes
 * slot q's per-element keys (myl7, in_bits q_bits[q], alpha thetas[4 i + q],
 * payload u64 1).
 * sufb200_trunc_bundle_eval_elem evaluates one party's n gates in one
 * launch, one element per thread: d_keys[q] (device) is slot q's key array
 * [n][key_bytes[q]], d_words (device) the party's words; d_y [n], d_bools
 * [n][3] or NULL. */
int sufb200_trunc_gen_elem(int kind, int frac_bits, uint64_t rng_seed, size_t n, sufb200_trunc_desc* shape0,
                           sufb200_trunc_desc* shape1, uint64_t* words0, uint64_t* words1, uint64_t* thetas,
                           uint64_t* r_in);
int sufb200_trunc_bundle_eval_elem(sufb200_ctx ctx, const sufb200_trunc_desc* shape, const uint8_t* const* d_keys,
                                   const size_t* key_bytes, const uint64_t* d_words, const uint64_t* d_xhat, size_t n,
                                   uint64_t* d_y, uint64_t* d_bools, void* stream);

/* The per-element keys of one slot rearranged level by level for the
 * evaluation kernel (an engine-internal device layout, made once per batch
 * of dealt keys): in blocks of 16,384 elements, the keys' seeds, per-level
 * correction words and final words as arrays over the block's elements, so
 * a warp reads one level of its 32 elements' keys as one coalesced run
 * instead of 32 records 33 in_bits + 40 bytes apart, a walk stays within a
 * few MB, and each key takes 25 in_bits + 24 bytes.
 * sufb200_elem_keys_soa_bytes gives the layout's size (0 for a bad width);
 * sufb200_elem_keys_to_soa fills it from d_keys [n][key_bytes] (adapter
 * layout, in_bits, party; d_soa 16-byte aligned; a key whose header does not
 * match is flagged through sufb200_ctx_sync and evaluates to 0);
 * sufb200_trunc_bundle_eval_elem_soa is sufb200_trunc_bundle_eval_elem over
 * those layouts (d_soa[q] per slot), with the same outputs. */
size_t sufb200_elem_keys_soa_bytes(int in_bits, size_t n);
int sufb200_elem_keys_to_soa(sufb200_ctx ctx, int in_bits, int party, const uint8_t* d_keys, size_t key_bytes,
                             size_t n, uint8_t* d_soa, void* stream);
int sufb200_trunc_bundle_eval_elem_soa(sufb200_ctx ctx, const sufb200_trunc_desc* shape, const uint8_t* const* d_soa,
                                       const uint64_t* d_words, const uint64_t* d_xhat, size_t n, uint64_t* d_y,
                                       uint64_t* d_bools, void* stream);

/* ---- composite tapes of truncation gates ----------------------------------
 * The serialized CompositePartyKey of gates::write_composite_tape /
 * read_composite_tape (include/gates/composite_fss.hpp:2458-2608), byte for
 * byte, for the gates composite_gen_trunc_gate deals (:645-833).
 * sufb200_trunc_write_tapes: composite_write_tapes (:2610) of the gate
 * sufb200_trunc_gen(kind, frac_bits, rng_seed) deals, keys0/keys1[q] the
 * parties' myl7 keys of its nkeys queries (sizes key_bytes[q]); bit_order is
 * the dealing backend's (proto::BitOrder: 0 MSB_FIRST, 1 LSB_FIRST).  Both
 * tapes have the same length, written to *len_out; tape0 = tape1 = NULL
 * queries it.  Either tape pointer may be NULL.
 * sufb200_trunc_read_tape: one party's tape of a gate of `kind` with mask
 * r_in (the compiled gate's, CompiledSUFGate::r_in) into a bundle descriptor
 * for sufb200_trunc_bundle_eval: desc gets the query plan and the shares,
 * key_off[q] / key_bytes[q] locate query q's key inside the tape (up to 4),
 * *r_in_share (may be NULL) the party's r_in share.  A tape that is not a
 * truncation gate's of that kind and mask returns SUFB200_ERR_KEY.
 * Per-element gates (sufb200_trunc_gen_elem material, on the device):
 * sufb200_trunc_write_tapes_elem writes element i's tape of one party at
 * d_out + i * stride (stride >= sufb200_trunc_tape_elem_stride) and its
 * length to d_len[i], one warp per element; d_r_in [n] are the elements'
 * masks (trunc_gen_elem's r_in), d_r_in_share [n] the party's r_in shares:
 * sufb200_trunc_gen_elem_rin_shares gives party 0's (party 1's = r_in -
 * party 0's). */
int sufb200_trunc_write_tapes(int kind, int frac_bits, uint64_t rng_seed, int bit_order, const uint8_t* const* keys0,
                              const uint8_t* const* keys1, const size_t* key_bytes, int nkeys, uint8_t* tape0,
                              uint8_t* tape1, size_t cap, size_t* len_out);
int sufb200_trunc_read_tape(const uint8_t* tape, size_t len, int kind, uint64_t r_in, int party,
                            sufb200_trunc_desc* desc, size_t* key_off, size_t* key_bytes, uint64_t* r_in_share);
int sufb200_trunc_gen_elem_rin_shares(int kind, int frac_bits, uint64_t rng_seed, size_t n, uint64_t* share0);
size_t sufb200_trunc_tape_elem_stride(const sufb200_trunc_desc* shape, const size_t* key_bytes);
int sufb200_trunc_write_tapes_elem(sufb200_ctx ctx, const sufb200_trunc_desc* shape, const uint8_t* const* d_keys,
                                   const size_t* key_bytes, const uint64_t* d_words, const uint64_t* d_r_in,
                                   const uint64_t* d_r_in_share, size_t n, int bit_order, uint8_t* d_out,
                                   size_t stride, uint64_t* d_len, void* stream);

/* Size of the fixed key staging array of sufb200_trunc_bundle_eval_noalloc. */
#define SUFB200_NOALLOC_KEY_BYTES 16384

/* Allocation-free form of sufb200_trunc_bundle_eval (no counterpart in the
 * reference; it exists for callers that cannot allocate device memory when
 * they evaluate -- a runtime that owns all device memory through its own
 * arena, or code that must not re-enter or grow the CUDA allocator).  The
 * bundle's keys are staged in one fixed array of SUFB200_NOALLOC_KEY_BYTES
 * (16 KiB; a valid bundle of four 64-bit-input keys needs 8640 bytes) that
 * every device loading the library holds until exit; the call makes no
 * cudaMalloc / cudaFree or other allocating call, and rejects
 * (SUFB200_ERR_INVALID) a bundle whose keys, each padded to 16 bytes, exceed
 * that size.  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current, and with CUDA's
 * lazy module loading it also loads the library's kernels, which allocates
 * device memory: make one call at set-up, before the phase that must not
 * allocate and before any stream capture.  The address stays cached for the
 * process: after cudaDeviceReset (or a re-created primary context) do not
 * call this entry point again.  All calls on a device share the array and it
 * keeps the last call's contents: calls whose copies and kernels overlap on
 * the GPU (different streams, no ordering) race with each other.  It always
 * runs the one-pass bundle kernel (the shared-prefix path of
 * sufb200_trunc_bundle_eval for n >= 16384 needs scratch sized by n), so it
 * is slower than that entry point on large batches; the outputs are the
 * same.  Arguments, checks and outputs are otherwise those of
 * sufb200_trunc_bundle_eval. */
int sufb200_trunc_bundle_eval_noalloc(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                                      const size_t* key_bytes, const uint64_t* d_xhat, size_t n, uint64_t* d_y,
                                      uint64_t* d_bools, void* stream);

/* ---- reference GPU-backend key formats (cuda/pfss_backend_gpu.cu) -------- */

/* Threshold "DCF" blob [in_bits u16][payload_len u16][alpha u64][payload]
 * (DcfKeyHeader, pfss_backend_gpu.cu:69-73,197-221); party 1 carries zeros.
 * Returns the blob size; writes it when out != NULL. */
size_t sufb200_thr_dcf_build(int in_bits, uint64_t alpha, const uint8_t* payload, int payload_len, uint8_t* out);

/* out = payload if (x & m) < (alpha & m) else 0 (eval_dcf_many_kernel
 * [_broadcast], pfss_backend_gpu.cu:386-433). */
int sufb200_thr_dcf_eval(sufb200_ctx ctx, int in_bits, const uint8_t* d_keys, size_t key_bytes, int broadcast,
                         const uint64_t* d_xs, size_t n, int out_bytes, void* d_out, void* stream);

/* Packed-compare blob (PackedCmpKeyHeader, 208 bytes + thresholds;
 * build_packed_cmp_key, pfss_backend_gpu.cu:257-288).  seed is 16 bytes. */
size_t sufb200_packed_lt_build(int party, uint64_t nonce, int in_bits, const uint64_t* thresholds, int num_thr,
                               const uint8_t* seed, uint8_t* out);

/* XOR-shared bitmasks 1[x < thr_j], AES-CTR masked with the kernel counter
 * layout ctr = nonce ^ (idx << 32) ^ (w/2), idx = idx_base + i
 * (packed_cmp_kernel_keyed[_broadcast], cuda/pfss_kernels.cu:240-423).
 * d_out is [n][out_words] u64. */
int sufb200_packed_lt_eval(sufb200_ctx ctx, const uint8_t* d_keys, size_t key_bytes, int broadcast,
                           const uint64_t* d_xs, size_t n, int in_bits, int out_words, uint64_t idx_base,
                           uint64_t* d_out, void* stream);

/* Interval-LUT blob (IntervalKeyHeader, 216 bytes + cuts + payload;
 * build_interval_key, pfss_backend_gpu.cu:223-255).  cuts has intervals+1
 * entries, payload intervals*out_words. */
size_t sufb200_interval_lut_build(int party, uint64_t nonce, int in_bits, int out_words, const uint64_t* cuts,
                                  int intervals, const uint64_t* payload, const uint8_t* seed, uint8_t* out);

/* Additive shares of the interval's payload row, AES-CTR masked with
 * ctr = nonce ^ (idx << 32) ^ (iv*out_words + w) (vector_lut_kernel_keyed
 * [_broadcast], cuda/pfss_kernels.cu:545-642).  d_out is [n][out_words]. */
int sufb200_interval_lut_eval(sufb200_ctx ctx, const uint8_t* d_keys, size_t key_bytes, int broadcast,
                              const uint64_t* d_xs, size_t n, int out_words, uint64_t idx_base, uint64_t* d_out,
                              void* stream);

/* myl7 DCF key pairs generated on the GPU, one per alpha: the same bytes as
 * sufb200_myl7_gen_batch (the reference's dcf_gen,
 * third_party/myl7_fss/src/dcf.c:42-142, in the adapter layout of
 * Myl7FssBackend::gen_dcf, include/proto/myl7_fss_backend.hpp:131-213) for
 * the same party seeds.  All arrays on the device: d_alphas [n],
 * d_seeds0/1 [n][16] (16-byte aligned), d_keys0/1 [n][key_bytes] (8-byte
 * aligned).  in_bits a multiple of 8 (8..64); payload 1..16 bytes, the same
 * for every key.  No counterpart in the reference, whose keygen runs on the
 * host. */
int sufb200_myl7_gen_batch_device(sufb200_ctx ctx, int group, int in_bits, const uint64_t* d_alphas, size_t n,
                                  const uint8_t* payload, int payload_len, const uint8_t* d_seeds0,
                                  const uint8_t* d_seeds1, uint8_t* d_keys0, uint8_t* d_keys1, void* stream);

/* Composite coefficient gate (ell = 0) in one pass: the coefficient words of
 * the interval containing x^ from a broadcast interval-LUT key (reference
 * IntervalKeyHeader blob, host memory, out_words = r * (degree + 1)), the
 * polynomial of each output over the public x^, and this party's output-mask
 * share: d_out[i*r + j] = sum_k c[j*(degree+1)+k] * x^^k + r_out[j] mod
 * 2^ring_bits.  degree 0 is the interval-LUT fast path of
 * composite_eval_batch_backend (include/gates/composite_fss.hpp:1253-1384:
 * eval_interval_lut_many_device_broadcast, then the r_out loop or
 * launch_add_rout_aos_kernel); degree > 0 its Horner-only path over x^
 * (composite_fss.hpp:2066-2130).  r <= 8; r_out may be NULL (zero masks). */
int sufb200_coeff_lut_eval(sufb200_ctx ctx, const uint8_t* key, size_t key_bytes, const uint64_t* d_xhat, size_t n,
                           int r, int degree, const uint64_t* r_out, int ring_bits, uint64_t idx_base,
                           uint64_t* d_out, void* stream);
/* Both parties' coefficient gates over the same public x^ in one launch (one
 * GPU holding both parties, as the reference's single-GPU runs do): party
 * 0's key / r_out0 / d_out0 and party 1's, the same r, degree and ring; each
 * output equals sufb200_coeff_lut_eval's for that party. */
int sufb200_coeff_lut_eval_pair(sufb200_ctx ctx, const uint8_t* key0, size_t key_bytes0, const uint8_t* key1,
                                size_t key_bytes1, const uint64_t* d_xhat, size_t n, int r, int degree,
                                const uint64_t* r_out0, const uint64_t* r_out1, int ring_bits, uint64_t idx_base,
                                uint64_t* d_out0, uint64_t* d_out1, void* stream);

/* seed_from_id (pfss_backend_gpu.cu:189-194): 16 bytes from
 * mt19937_64(id ^ tweak * 0x9e3779b97f4a7c15). */
int sufb200_seed_from_id(uint64_t id, uint64_t tweak, uint8_t* seed16);

/* ---- elementwise / row primitives (include/runtime/cuda_primitives.hpp) -- */

/* z = c + d*b + e*a (+ d*e on party 0) mod 2^64 (launch_beaver_mul_kernel). */
int sufb200_beaver_mul(int party, const uint64_t* d_a, const uint64_t* d_b, const uint64_t* d_c,
                       const uint64_t* d_d_open, const uint64_t* d_e_open, uint64_t* d_out, size_t n, void* stream);

/* Same with {a,b,c} triples interleaved (launch_beaver_mul_aos_kernel). */
int sufb200_beaver_mul_aos(int party, const uint64_t* d_triples, const uint64_t* d_d_open,
                           const uint64_t* d_e_open, uint64_t* d_out, size_t n, void* stream);

/* ((c3*x + c2)*x + c1)*x + c0 mod 2^64 (launch_horner_cubic_kernel). */
int sufb200_horner_cubic(const uint64_t* d_x, const uint64_t* d_c0, const uint64_t* d_c1, const uint64_t* d_c2,
                         const uint64_t* d_c3, uint64_t* d_out, size_t n, void* stream);

/* Truncation postproc (launch_trunc_postproc_kernel): kind_gapars 0 =
 * faithful (sign_idx < 0 for TR, >= 0 for ARS), 1 = GapARS. */
int sufb200_trunc_postproc(int party, int kind_gapars, int frac_bits, uint64_t r_hi_share, uint64_t m_share,
                           const uint64_t* d_hatx, const uint64_t* d_arith, size_t arith_stride, int arith_idx,
                           const uint64_t* d_bools, size_t bool_stride, int carry_idx, int sign_idx, int wrap_idx,
                           uint64_t* d_out, size_t n, void* stream);

/* out[i*out_words + j] += r_out[j], r_out in host memory, out_words <= 8
 * (launch_add_rout_aos_kernel). */
int sufb200_add_rout_aos(uint64_t* d_out, size_t elems, int out_words, const uint64_t* r_out, size_t r_out_words,
                         void* stream);

/* Per-row sums mod 2^64, optional valid lengths (launch_row_sum_kernel). */
int sufb200_row_sum(const uint64_t* d_mat, int rows, int cols, const int* d_valid_lens, uint64_t* d_out_rows,
                    void* stream);

/* Ragged rows back to back, offsets[rows+1] (launch_row_sum_ragged_kernel). */
int sufb200_row_sum_ragged(const uint64_t* d_vals, const int* d_row_offsets, int rows, uint64_t* d_out_rows,
                           void* stream);

/* sum (x - mean)^2 per row (launch_row_variance_kernel). */
int sufb200_row_variance(const uint64_t* d_mat, const uint64_t* d_mean, int rows, int cols, const int* d_valid_lens,
                         uint64_t* d_out_rows, void* stream);

/* Row-broadcast Beaver mul (launch_row_broadcast_mul_kernel). */
int sufb200_row_broadcast_mul(int party, const uint64_t* d_A, const uint64_t* d_B_rows, const uint64_t* d_C,
                              const uint64_t* d_d_open, const uint64_t* d_e_open_rows, int rows, int cols,
                              const int* d_valid_lens, uint64_t* d_out, void* stream);

/* Dense bitstream of eff_bits-wide values (launch_pack_eff_bits_kernel /
 * launch_unpack_eff_bits_kernel); packed has ceil(n*eff_bits/64) words. */
int sufb200_pack_eff_bits(const uint64_t* d_in, int eff_bits, uint64_t* d_packed, size_t n, void* stream);
int sufb200_unpack_eff_bits(const uint64_t* d_packed, int eff_bits, uint64_t* d_out, size_t n, void* stream);

/* Open: unpack remote packed share, add local, mask to ring_bits
 * (launch_unpack_add_mod_kernel). */
int sufb200_unpack_add_mod(const uint64_t* d_local, const uint64_t* d_packed_remote, int eff_bits, uint64_t* d_out,
                           size_t n, int ring_bits, void* stream);

/* Unpack, add local and sign-extend to ring_bits
 * (launch_unpack_add_to_signed_kernel). */
int sufb200_unpack_add_to_signed(const uint64_t* d_local, const uint64_t* d_packed_remote, int eff_bits,
                                 uint64_t* d_out, size_t n, int ring_bits, void* stream);

/* ---- paired-GPU open ------------------------------------------------------
 * Replaces the exchange of OpenCollector::flush
 * (src/runtime/open_collector.cpp:357-895), which packs a flush, moves it
 * device -> host -> net::Chan -> host -> device and adds the peer's words:
 * here the two parties' GPUs (party 0 on GPU j, party 1 on GPU j + N/2)
 * swap the packed words over NVLink in one NCCL group call, enqueued with the
 * pack and the add on the caller's stream.
 *
 * sufb200_open_unique_id writes the 128-byte NCCL id on one rank; the caller
 * hands it to the others out of band.  sufb200_open_comm_create joins the
 * communicator (all nranks ranks call it) and returns SUFB200_ERR_COMM if the
 * peers have not all joined within timeout_s seconds.  sufb200_open_exchange:
 * both ranks of a pair call it with the same n, eff_bits and ring_bits;
 * d_out = local + peer (mod 2^ring_bits; sign-extended from ring_bits when
 * signed_out) for the low eff_bits of every share (eff_bits = 64 sends the
 * raw words).  If a peer stops calling, its partner's exchange never
 * completes on the GPU: sufb200_open_comm_abort (from any thread) ends it. */
#define SUFB200_OPEN_ID_BYTES 128
typedef struct sufb200_open_comm_s* sufb200_open_comm;
int sufb200_open_unique_id(uint8_t* id);
int sufb200_open_comm_create(sufb200_ctx ctx, const uint8_t* id, int nranks, int rank, double timeout_s,
                             sufb200_open_comm* out);
int sufb200_open_comm_destroy(sufb200_open_comm comm);
int sufb200_open_comm_abort(sufb200_open_comm comm);
int sufb200_open_exchange(sufb200_open_comm comm, int peer, const uint64_t* d_local, size_t n, int eff_bits,
                          int ring_bits, int signed_out, uint64_t* d_out, void* stream);

/* ---- paired-GPU open in one kernel (peer stores over NVLink) ---------------
 * The same exchange as sufb200_open_exchange, fused: one kernel packs this
 * rank's shares to eff_bits-wide words (the pack_eff_bits wire format of
 * OpenCollector::flush, src/runtime/open_collector.cpp:357-895,
 * cuda/pfss_kernels.cu:722-812), stores them straight into the paired GPU's
 * landing buffer, raises a per-CTA flag there, waits for the peer's flag and
 * writes d_out = local + peer (mod 2^ring_bits, sign-extended when
 * signed_out).  sufb200_p2p_open_create allocates this rank's landing buffer
 * (room for max_words packed words per call, cudaMalloc) and writes the
 * SUFB200_P2P_HANDLE_BYTES blob the peer passes to sufb200_p2p_open_connect
 * (out of band).  Both ranks call exchange with the same n / eff_bits /
 * ring_bits, on one stream each, in the same order.  Waits are bounded by
 * timeout_s: a peer that does not call ends the kernel with
 * SUFB200_ERR_CUDA from sufb200_ctx_sync (status: timeout) and d_out
 * undefined.  The two ranks must be on different GPUs (connect refuses a
 * peer on the same device).
 * sufb200_p2p_open_connect_self instead makes the endpoint its own peer (a
 * single-device check of the whole kernel: each CTA waits only on the flag
 * it raised itself); exchange then writes d_out = local + (local mod
 * 2^eff_bits), reduced and sign-extended as above. */
#define SUFB200_P2P_HANDLE_BYTES 128
typedef struct sufb200_p2p_open_s* sufb200_p2p_open;
int sufb200_p2p_open_create(sufb200_ctx ctx, size_t max_words, sufb200_p2p_open* out, uint8_t* handle_out);
int sufb200_p2p_open_connect(sufb200_p2p_open h, const uint8_t* peer_handle);
int sufb200_p2p_open_connect_self(sufb200_p2p_open h);
int sufb200_p2p_open_exchange(sufb200_p2p_open h, const uint64_t* d_local, size_t n, int eff_bits, int ring_bits,
                              int signed_out, uint64_t* d_out, double timeout_s, void* stream);
int sufb200_p2p_open_destroy(sufb200_p2p_open h);

/* local + remote, sign-extended to ring_bits (launch_open_add_to_signed_kernel). */
int sufb200_open_add_to_signed(const uint64_t* d_local, const uint64_t* d_remote, uint64_t* d_out, size_t n,
                               int ring_bits, void* stream);

/* ---- ring matmuls on the tensor cores -------------------------------------
 * Exact Z_2^64 products by 8-bit limbs on tcgen05 (36 limb products per
 * 32-deep step, int32 accumulators per limb diagonal in tensor memory);
 * the contraction depth (2K for the Beaver form) must not exceed 8192.
 * Both report a kernel-side timeout through sufb200_ctx_sync.
 *
 * sufb200_ring_matmul: matmul_publicW_gpu / matmul_publicW_tiled
 * (src/nn/matmul_gpu.cu:21-117, 388-420): Y[b] = X[b] W (+ bias per column)
 * mod 2^64, X [batch][M][K] shares, W [K][N] (or [N][K] when w_transposed)
 * public int64, bias [N] or NULL.
 * sufb200_beaver_matmul2d_tc: the same results as sufb200_beaver_matmul2d
 * (launch_beaver_matmul2d[_batched]_kernel, cuda/cuda_primitives.cu:391-628),
 * computed as one product [D | A] x [B (+ E for party 0) ; E] plus C. */
int sufb200_ring_matmul(sufb200_ctx ctx, const uint64_t* d_x, const int64_t* d_w, const int64_t* d_bias,
                        uint64_t* d_y, size_t batch, int M, int K, int N, int w_transposed, void* stream);
int sufb200_beaver_matmul2d_tc(sufb200_ctx ctx, int party, const uint64_t* d_D_open, const uint64_t* d_E_open,
                               const uint64_t* d_A, const uint64_t* d_B, const uint64_t* d_C, int batches, int M,
                               int K, int N, int w_transposed, int has_scale, int64_t mul_const, int mul_shift,
                               uint64_t* d_out, void* stream);

/* Row mean = row sum / len, unsigned (launch_row_mean_kernel). */
int sufb200_row_mean(const uint64_t* d_mat, int rows, int cols, const int* d_valid_lens, uint64_t* d_out_rows,
                     void* stream);

/* x >> frac_bits (launch_trunc_shift_kernel). */
int sufb200_trunc_shift(const uint64_t* d_in, uint64_t* d_out, int frac_bits, size_t n, void* stream);

/* Beaver matmul out = C + D*B + A*E (+ D*E on party 0) mod 2^64 for
 * `batches` instances sharing the triple (A [MxK], B [KxN] or [NxK] when
 * w_transposed, C [MxN]); D, E, out per instance.  With has_scale, each
 * output is the low word of (int128)(int64)acc * mul_const >> mul_shift
 * (launch_beaver_matmul2d[_batched]_kernel, cuda/cuda_primitives.cu:391-628). */
int sufb200_beaver_matmul2d(int party, const uint64_t* d_D_open, const uint64_t* d_E_open, const uint64_t* d_A,
                            const uint64_t* d_B, const uint64_t* d_C, int batches, int M, int K, int N,
                            int w_transposed, int has_scale, int64_t mul_const, int mul_shift, uint64_t* d_out,
                            void* stream);

/* ---- configs[4] softmax block, device-resident --------------------------- */

/* The seven truncations of the block, in order: nExp T_f(p), the first T_f
 * of the nExp T_2f(r), reciprocal init, Newton T_f(y s), Newton T_f(y d),
 * probability T_f, and the second T_f of T_2f(r).  CubicPolyTask's T_2f is
 * done as T_f(T_f(r)): floor(floor(r / 2^f) / 2^f) = floor(r / 2^2f), so the
 * result is the same word, and each half is an f-bit GapARS bundle (a
 * full-domain table lookup) instead of a 2f-bit one (a walk of f levels per
 * element past the shared prefix). */
#define SUFB200_SOFTMAX_TRUNCS 7

/* One party's dealer material for sufb200_softmax_block_pair.  Every triple
 * array holds (a, b, c) words interleaved; the interval-LUT keys are device
 * copies of broadcast IntervalKeyHeader blobs with 4 coefficient words per
 * interval, built on the x^ = x + r_in domain of their gate. */
typedef struct sufb200_softmax_party {
  uint64_t nexp_rin, recip_rin;   /* this party's shares of the LUT gates' r_in */
  const uint8_t* d_nexp_lut;      /* device */
  size_t nexp_lut_bytes;
  const uint8_t* d_recip_lut;     /* device */
  size_t recip_lut_bytes;
  const uint64_t* d_nexp_triples; /* device [3][n][3]: c3*t, u*t, q*t */
  const uint64_t* d_recip_triples;/* device [3][rows][3]: a1*s, y*s, y*d */
  const uint64_t* d_row_a;        /* device [n]   row-broadcast triple A */
  const uint64_t* d_row_b;        /* device [rows] B */
  const uint64_t* d_row_c;        /* device [n]   C = A * B[row] */
  sufb200_trunc_desc trunc[SUFB200_SOFTMAX_TRUNCS];
  uint64_t trunc_rin[SUFB200_SOFTMAX_TRUNCS];              /* shares of each truncation's r_in */
  const uint8_t* trunc_keys[SUFB200_SOFTMAX_TRUNCS][4];    /* myl7 key of each query: host, or device */
  size_t trunc_key_bytes[SUFB200_SOFTMAX_TRUNCS][4];
  int32_t trunc_keys_device;  /* nonzero: trunc_keys are device pointers (resident; no copy per call) */
  /* device, or NULL: bundle k's tables (sufb200_trunc_tables_dev over this
   * party's device keys).  With device keys and both parties' tables set,
   * the block evaluates bundle k against them instead of walking its keys. */
  const void* trunc_tables[SUFB200_SOFTMAX_TRUNCS];
  /* cudaEvent_t or NULL: the block makes its stream wait for this event
   * right before it reads bundle k's tables (tables filled on another
   * stream while the block's earlier steps run).  Read from party 0. */
  void* trunc_ready[SUFB200_SOFTMAX_TRUNCS];
} sufb200_softmax_party;

/* nn::SoftmaxBlockTask (include/nn/softmax_block_task.hpp) for BOTH parties
 * on one GPU, every open computed on the device: nExp cubic gate
 * (CubicPolyTask, include/runtime/phase_tasks.hpp:2670-3140), ragged row sums,
 * reciprocal with one Newton step (RecipTask, :3140-3650), row-broadcast
 * Beaver product and probability truncation.  t0/t1: the parties' shares of
 * the packed active max-differences (Q frac_bits), n = row_off[rows];
 * row_off: device [rows + 1].  prob0/prob1: shares of the packed
 * probabilities.  Asynchronous on `stream`; 24 launches, no host sync. */
int sufb200_softmax_block_pair(sufb200_ctx ctx, const sufb200_softmax_party* p0, const sufb200_softmax_party* p1,
                               int rows, const int32_t* d_row_off, const uint64_t* d_t0, const uint64_t* d_t1,
                               size_t n, int frac_bits, uint64_t* d_prob0, uint64_t* d_prob1, void* stream);

/* The eight truncations of the LayerNorm block, in order: mean T_f, variance
 * T_2f, rsqrt init T_f(c1 v), T_f(y y), T_f(v y2), the halving T_1(x y2),
 * the Newton update T_f(y t), the normalised output T_f(d y). */
#define SUFB200_LAYERNORM_TRUNCS 8

/* One party's dealer material for sufb200_layernorm_block_pair (rows x cols,
 * dense).  Triple arrays hold (a, b, c) interleaved. */
typedef struct sufb200_layernorm_party {
  uint64_t rsqrt_rin;              /* this party's share of the rsqrt LUT gate's r_in */
  const uint8_t* d_rsqrt_lut;      /* device: broadcast IntervalKeyHeader blob, 4 words per interval */
  size_t rsqrt_lut_bytes;
  const uint64_t* d_sq_triples;    /* device [rows*cols][3]: d * d */
  const uint64_t* d_row_triples;   /* device [4][rows][3]: c1*v, y*y, v*y2, y*t */
  const uint64_t* d_norm_a;        /* device [rows*cols] row-broadcast triple A */
  const uint64_t* d_norm_b;        /* device [rows] B */
  const uint64_t* d_norm_c;        /* device [rows*cols] C = A * B[row] */
  sufb200_trunc_desc trunc[SUFB200_LAYERNORM_TRUNCS];
  uint64_t trunc_rin[SUFB200_LAYERNORM_TRUNCS];
  const uint8_t* trunc_keys[SUFB200_LAYERNORM_TRUNCS][4]; /* host, or device (trunc_keys_device) */
  size_t trunc_key_bytes[SUFB200_LAYERNORM_TRUNCS][4];
  int32_t trunc_keys_device;  /* nonzero: trunc_keys are device pointers */
  const void* trunc_tables[SUFB200_LAYERNORM_TRUNCS]; /* device or NULL, as in sufb200_softmax_party */
  void* trunc_ready[SUFB200_LAYERNORM_TRUNCS];        /* cudaEvent_t or NULL, as in sufb200_softmax_party */
} sufb200_layernorm_party;

/* runtime::LayerNormTask with RsqrtTask (include/runtime/phase_tasks.hpp:
 * 1383-1700, 2186-2600; one Newton step, no affine) for BOTH parties on one
 * GPU, every open on the device, computed with Beaver products and
 * truncation bundles throughout:
 *   mu = T_f(sum x * inv_len), d = x - mu, v = T_2f(sum d^2 * inv_len) + eps,
 *   y = c0 + T_f(c1 v) with (c0, c1) = LUT_rsqrt(v),
 *   y = T_f(y (3 2^(f-1) - T_1(T_f(v T_f(y y))))), out = T_f(d y[row]).
 * (The reference's RsqrtTask forms its initial guess from the opened input
 * and halves x y^2 with a local shift of each share; on additive shares both
 * are replaced here by the secure steps above, which compute the same
 * fixed-point function.)  inv_len and eps are public Q(frac_bits) constants;
 * eps is added once.  x0/x1: [rows*cols] shares; out0/out1 likewise.
 * Asynchronous on `stream`. */
int sufb200_layernorm_block_pair(sufb200_ctx ctx, const sufb200_layernorm_party* p0,
                                 const sufb200_layernorm_party* p1, int rows, int cols, const uint64_t* d_x0,
                                 const uint64_t* d_x1, int frac_bits, uint64_t inv_len, uint64_t eps,
                                 uint64_t* d_out0, uint64_t* d_out1, void* stream);

/* ---- host utilities ----------------------------------------------------- */

/* ---- glue of the device-resident transformer layer (both parties, one GPU) --
 * Every party's share is computed from that party's own material; where the
 * protocol opens a masked value, the open is the sum of both parties'
 * masked shares (OpenCollector::flush, src/runtime/open_collector.cpp:357-895,
 * with both shares at hand).
 *
 * sufb200_open_masked_pair: x^ = (a0 + r0) + (a1 + r1), the masked input of
 * the gate after a local product (TruncTask / CubicPolyTask open of x + r_in,
 * include/runtime/phase_tasks.hpp).
 * sufb200_add_pair: out_p = a_p + b_p (residual adds).
 * sufb200_relu_open_pair / sufb200_relu_update_pair: one round of the row-max
 * tournament of nn::RowMaxDiffTask (include/nn/row_maxdiff_task.hpp):
 * x^[r][j] = sum_p (c_p[r][2j] - c_p[r][2j+1] + r_p) opens the difference for
 * the ReLU gate; next_p[r][j] = c_p[r][2j+1] + relu_p[r][j] = max in shares.
 * sufb200_maxdiff_pair: t_p[r][c] = max_p[r] - x_p[r][c].
 * sufb200_beaver_open_pair: per head h < heads, both parties' Beaver matmul
 * shares Z_p = C_p + D B_p + A_p E (+ D E for party 0), D = X - A and E = Y - B
 * opened from the parties' shares (nn::matmul_beaver, launch_beaver_matmul2d_kernel,
 * cuda/cuda_primitives.cu:391-628), written as the open of the masked result
 * out(h, m, n) = sum_p (Z_p + r[p]).  d_x[p], d_y[p], d_a[p], d_b[p], d_c[p] are
 * two-entry host arrays of device pointers; X (h, m, k) at x + h*sx + m*ldx + k,
 * Y (h, k, n) at y + h*sy + k*ldy + n (y_transposed: n*ldy + k), A [heads][M][K],
 * B [heads][K][N] ([heads][N][K] transposed), C [heads][M][N] contiguous; out
 * (h, m, n) at d_out + h*so + m*ldo + n. */
int sufb200_open_masked_pair(const uint64_t* d_a0, const uint64_t* d_a1, uint64_t r0, uint64_t r1, uint64_t* d_xhat,
                             size_t n, void* stream);
int sufb200_add_pair(const uint64_t* d_a0, const uint64_t* d_b0, const uint64_t* d_a1, const uint64_t* d_b1,
                     uint64_t* d_out0, uint64_t* d_out1, size_t n, void* stream);
int sufb200_relu_open_pair(const uint64_t* d_c0, const uint64_t* d_c1, int rows, int width, uint64_t r0, uint64_t r1,
                           uint64_t* d_xhat, void* stream);
int sufb200_relu_update_pair(const uint64_t* d_c0, const uint64_t* d_c1, const uint64_t* d_relu0,
                             const uint64_t* d_relu1, int rows, int width, uint64_t* d_next0, uint64_t* d_next1,
                             void* stream);
int sufb200_maxdiff_pair(const uint64_t* d_max0, const uint64_t* d_max1, const uint64_t* d_x0, const uint64_t* d_x1,
                         int rows, int cols, uint64_t* d_t0, uint64_t* d_t1, void* stream);
int sufb200_beaver_open_pair(const uint64_t* const* d_x, size_t sx, int ldx, const uint64_t* const* d_y, size_t sy,
                             int ldy, int y_transposed, const uint64_t* const* d_a, const uint64_t* const* d_b,
                             const uint64_t* const* d_c, const uint64_t* r, int heads, int M, int K, int N,
                             uint64_t* d_out, size_t so, int ldo, void* stream);

/* n successive draws of mt19937_64(seed) (the reference's mask / key RNG). */
int sufb200_host_mt19937_64(uint64_t seed, uint64_t* out, size_t n);

#ifdef __cplusplus
}
#endif

#endif /* SUFB200_H_ */
