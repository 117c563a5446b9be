/*
 * kq.h -- the C ABI of the B200 Q4_K / Q6_K matvec library (libkq.so).
 *
 * This is the drop-in boundary. fxeqxmulfx/kernite calls a kernel through a macro-generated
 * launcher `unsafe fn <kernel>(&self, grid: Grid, params...) -> Result<(), kernite_cuda::Error>`
 * (crates/macros/src/gpu.rs:276-328) on a `Kernels` struct that `Kernels::load(&Cuda)` fills by
 * loading a module (crates/macros/src/gpu.rs:74-98, crates/cuda/src/lib.rs:945-1016), and
 * launches with `cuLaunchKernel` (crates/cuda/src/lib.rs:1045-1054). Each entry point below
 * replaces one piece of that, as its comment says.
 *
 * Conventions (kernite-cuda's, kept):
 *  - Device pointers are plain 64-bit addresses, exactly what `kernite_cuda::Ptr::addr()`
 *    gives (crates/cuda/src/lib.rs:776-837). The library never owns a caller's buffer.
 *  - Every entry point returns 0 on success, or an error code: a CUDA error number (< 1000),
 *    or one of KQ_E_* below. kq_last_error() then gives the thread's last error as
 *    "<call>: <NAME> (<n>): <meaning>[: detail]", the shape of kernite_cuda::Error's Display
 *    (crates/cuda/src/lib.rs:290-324). Arguments are checked before any launch; a bad
 *    argument is KQ_E_INVALID, never a device fault.
 *  - Launches are asynchronous on the given stream (NULL = the legacy default stream, on which
 *    kernite launches everything, crates/cuda/src/lib.rs:1051).
 *  - A kq_ctx is for the thread and GPU that made it, as a kernite `Cuda` is
 *    (crates/cuda/src/lib.rs:27-35). kq_ctx_create leaves its device current, as Cuda::on makes
 *    its context current; every other entry point makes the ctx's device current for the call
 *    if it is not, and makes the caller's device current again before it returns.
 *  - Each kq_ctx has its own device error word: errors recorded by one ctx's launches are read
 *    and cleared by kq_device_error on that ctx only.
 *
 * Safety contract (kernite's launcher contract, crates/cuda/src/lib.rs:1035-1044): every pointer
 * must be device memory of the ctx's GPU, valid until the launch completes; the host must not
 * touch memory a launch writes until it completes.
 *
 * Formats: Q4_K super-block = 144 bytes {fp16 d, fp16 dmin, u8 scales[12], u8 qs[128]};
 * Q6_K super-block = 210 bytes {u8 ql[128], u8 qh[64], i8 scales[16], fp16 d}; 256 weights
 * each (GGML k-quant layout). A matrix of `rows` x `k` is rows * (k/256) consecutive blocks,
 * row-major.
 */
#ifndef KQ_H
#define KQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KQ_ABI_VERSION 1

enum {
    KQ_OK = 0,
    KQ_E_INVALID = 1001,     /* an argument was rejected before launch */
    KQ_E_UNSUPPORTED = 1002, /* a valid request this build does not serve (e.g. a shape limit) */
    KQ_E_DEVICE = 1003,      /* the device reported a failed bounded wait (see kq_device_error) */
    KQ_E_COMM = 1004         /* a multi-GPU exchange failed */
};

/* Quantisation types, GGML's type numbers. */
enum { KQ_TYPE_Q4_K = 12, KQ_TYPE_Q5_K = 13, KQ_TYPE_Q6_K = 14 };
/* More types: decoded (kq_dequant_*) and multiplied by kq_matvec at batch 1 without prologue or
 * epilogue, on the CUDA cores (k * 4 bytes of x must fit in shared memory). Q2_K: 84-byte blocks
 * of 256; Q3_K: 110-byte blocks of 256 (rows 2-byte aligned); Q8_0: 34-byte blocks of 32 (a row
 * of k weights is k / 32 blocks, k a multiple of 256). W 16-byte aligned for all. */
enum { KQ_TYPE_Q8_0 = 8, KQ_TYPE_Q2_K = 10, KQ_TYPE_Q3_K = 11 };

/* What a matvec does to x before the product, and to each output after it. */
enum { KQ_PROLOGUE_NONE = 0, KQ_PROLOGUE_RMSNORM = 1 };
enum { KQ_EPILOGUE_NONE = 0, KQ_EPILOGUE_PAIR_PRODUCT = 1, KQ_EPILOGUE_SILU_PRODUCT = 2 };

/* Flags for kq_matvec_desc.flags. */
enum {
    /* The weights were written before the previous kernel on the stream began: the kernel may
     * start streaming them before that kernel ends (programmatic dependent launch). */
    KQ_FLAG_WEIGHTS_STATIC = 1u << 0,
    /* Launch without the programmatic-dependent-launch attribute. */
    KQ_FLAG_NO_PDL = 1u << 1,
    /* Use the tensor-core (tcgen05) kernel; Q4_K and Q5_K. */
    KQ_FLAG_TENSOR_CORES = 1u << 2,
    /* Use the CUDA-core kernel (batch <= 8, f32 multiply-adds). */
    KQ_FLAG_CUDA_CORES = 1u << 3,
    /* Use the warp-MMA kernel (Q4_K batch 1..8, Q5_K and Q6_K batch 1): dequantisation in
     * registers into exact tensor-core operands (integer at batch 1, f16 above), products
     * through mma.sync, f32 accumulation.
     * Without a path flag the library chooses: warp-MMA where it serves the request, the
     * tensor-core kernel above batch 8 (Q5_K: above batch 1), the CUDA-core kernel otherwise. */
    KQ_FLAG_WARP_MMA = 1u << 4
    /* Bits 29 and 30 are reserved for the library's tests and A/B timing: on the warp-MMA path
     * they select its other operand variant at batch 1 (f16 instead of integer) and its other
     * warp arrangement. Results stay within the same tolerance; callers leave them clear. */
};

typedef struct kq_ctx kq_ctx;
typedef void* kq_stream; /* a cudaStream_t / CUstream; NULL = legacy default stream */

/* Opens GPU `device`: retains its primary context (the one kernite-cuda's Cuda::on retains,
 * crates/cuda/src/lib.rs:570-617, so buffers from kernite's Cuda::alloc are valid here), reads
 * its attributes and prepares every kernel of the library. Replaces Cuda::on(i) followed by the
 * macro's Kernels::load(&cuda) (crates/macros/src/gpu.rs:74-98). */
int kq_ctx_create(int device, kq_ctx** out);

/* Frees what the ctx owns. Replaces `Drop for Module` (crates/cuda/src/lib.rs:1129-1138). */
int kq_ctx_destroy(kq_ctx* ctx);

/* The calling thread's last error, NUL-terminated into buf (truncated to len). Returns the
 * full length. Replaces kernite_cuda::Error's Display (crates/cuda/src/lib.rs:290-324). */
size_t kq_last_error(char* buf, size_t len);

/* The ctx's GPU: its ordinal, SM count and opt-in shared memory per block. Replaces
 * Cuda::multiprocessors / max_shared (crates/cuda/src/lib.rs:602-631). */
int kq_ctx_info(const kq_ctx* ctx, int* device, int* sm_count, int* max_smem_per_block);

/* Waits for the ctx's device, then reads and clears the device error word that the kernels'
 * bounded waits set instead of hanging. 0 if clear, KQ_E_DEVICE (with a message naming the
 * wait) if a kernel gave up. No reference counterpart: kernite's kernels have no bounded waits. */
int kq_device_error(kq_ctx* ctx);

/* y[b*rows + r] = sum_k W[r,k] * x[b*k + k'] for b < batch, r < rows: the Q4_K matvec.
 * batch 1..64 (above 8 on the tensor cores). W: 16-byte aligned; x: 16-byte aligned f32; y: f32.
 * Replaces a macro launcher `kernels.matvec_q4k(grid, y, w, x, rows, k)` of kernite's shape
 * (crates/macros/src/gpu.rs:276-328); the grid is the library's choice, not the caller's. */
int kq_matvec_q4k(kq_ctx* ctx, uint64_t y, uint64_t w, uint64_t x, uint32_t rows, uint32_t k,
                  uint32_t batch, kq_stream stream);

/* The same for Q6_K (210-byte blocks; rows may start at any even byte offset); batch 1..8. */
int kq_matvec_q6k(kq_ctx* ctx, uint64_t y, uint64_t w, uint64_t x, uint32_t rows, uint32_t k,
                  uint32_t batch, kq_stream stream);

/* The general form: strides, fused prologue/epilogue, flags. */
typedef struct kq_matvec_desc {
    uint32_t type;     /* KQ_TYPE_Q4_K, KQ_TYPE_Q5_K, KQ_TYPE_Q6_K (or Q2_K, Q3_K, Q8_0 below);
                        * Q5_K: batch 1 on the warp-MMA kernel, 2..64 on the tensor cores, no
                        * CUDA-core kernel */
    uint32_t rows, k;  /* W is rows x k; k % 256 == 0 */
    uint32_t batch;    /* vectors: 1..64 for Q4_K and Q5_K, 1..8 for Q6_K */
    uint64_t y, w, x;  /* device addresses */
    uint64_t ldx;      /* floats between vectors of x (>= k, multiple of 4); 0 = k */
    uint64_t ldy;      /* floats between vectors of y; 0 = rows (or rows/2 for the products) */
    uint32_t prologue; /* KQ_PROLOGUE_*: RMSNORM uses x / sqrt(mean(x^2) + eps) */
    uint32_t epilogue; /* KQ_EPILOGUE_*: PAIR_PRODUCT writes y[r/2] = v(r) * v(r+1) * pair_scale
                          for even r (rows must be even); SILU_PRODUCT writes
                          y[r/2] = silu(v(r)) * v(r+1) * pair_scale, silu(z) = z / (1 + e^-z):
                          a gated FFN's gate and up rows interleaved, as Llama's SiLU(W_gate x)
                          * (W_up x) */
    float eps;
    float pair_scale;
    uint32_t flags;    /* KQ_FLAG_* */
    uint32_t reserved;
} kq_matvec_desc;

/* Replaces the same launcher as kq_matvec_q4k, with kernite's per-kernel instance choice
 * (examples/matmul/src/gpu.rs:360-391) made from the descriptor. */
int kq_matvec(kq_ctx* ctx, const kq_matvec_desc* desc, kq_stream stream);

/* kq_matvec with x and y in host memory, for callers that hold their vectors on the host (as a
 * kernite caller does around Buffer::copy_from_host / copy_to_host, crates/cuda/src/lib.rs):
 * copies x (batch rows of ldx floats) into the context's device staging buffer, runs the matvec
 * with desc->w on the device, and copies y (batch rows of the output, ldy floats apart) back,
 * all on `stream`; synchronise the stream before reading y. desc->x and desc->y are ignored.
 * Page-locked host memory makes the copies asynchronous. The staging buffer grows on demand
 * (cudaMalloc: not inside a stream capture); calls that may overlap on the GPU need separate
 * contexts. */
int kq_matvec_host(kq_ctx* ctx, const kq_matvec_desc* desc, float* y_host, const float* x_host,
                   kq_stream stream);

/* out[256*i + e] = weight e of block i, for nblocks blocks at w, in the canonical order
 * w = (f32(d)*f32(sc))*f32(q) - f32(dmin)*f32(m) (Q4_K) / (f32(d)*f32(scale))*f32(q-32) (Q6_K),
 * each operation rounded to f32: bit-exact with the CPU decode. A verification kernel. No
 * reference counterpart (kernite has no k-quant decode); its bit-exact discipline follows
 * examples/matmul/src/reference.rs:1-10. */
int kq_dequant_q4k(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream);
int kq_dequant_q6k(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream);
/* Q5_K (176-byte blocks {fp16 d, fp16 dmin, u8 scales[12], u8 qh[32], u8 qs[128]}, 16-byte
 * aligned w): Q4_K's decode with q = nibble | fifth bit << 4, the fifth bit of element 32g + l
 * in bit g of qh[l]. */
int kq_dequant_q5k(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream);
/* Q2_K (84-byte blocks {u8 scales[16], u8 qs[64], fp16 d, fp16 dmin}): element 128h + 32s + l
 * is bits 2s..2s+1 of qs[32h + l], sub-block e/16 has scale (low nibble) and min (high nibble)
 * scales[e/16]; w = (f32(d)*f32(sc))*f32(q) - f32(dmin)*f32(m). */
int kq_dequant_q2k(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream);
/* Q3_K (110-byte blocks {u8 hmask[32], u8 qs[64], u8 scales[12], fp16 d}): q = bits 2s..2s+1
 * of qs[32h + l], minus 4 unless bit 4h + s of hmask[l] is set; sixteen 6-bit scales stored + 32;
 * w = (f32(d)*f32(scale))*f32(q). */
int kq_dequant_q3k(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream);
/* Q8_0, counted in units of eight 34-byte blocks {fp16 d, i8 qs[32]} (256 weights, 272 bytes):
 * w = f32(q) * f32(d). nblocks = units. */
int kq_dequant_q8_0(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream);

/* Writes synthetic blocks [block0, block0 + nblocks) of the tensor whose stream key is `key`
 * at w (w points at block0): counter-based splitmix64, so any range is reproducible on the CPU.
 * Q4_K: scale/quant bytes uniform, d and dmin = fp16(uniform[2^-10, 2^-6]); Q6_K: ql/qh bytes
 * uniform, scales uniform in [-64, 63], d = fp16(uniform[2^-12, 2^-8]). Stands in for the
 * seeded xorshift inputs of examples/matmul/src/main.rs:116-125. */
int kq_fill_q4k(kq_ctx* ctx, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
                kq_stream stream);
int kq_fill_q6k(kq_ctx* ctx, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
                kq_stream stream);
/* Q5_K: scale/qh/quant bytes uniform, d and dmin = fp16(uniform[2^-11, 2^-7]). */
int kq_fill_q5k(kq_ctx* ctx, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
                kq_stream stream);

/* The stream key of tensor `tensor` under `seed` (host function; the same as the oracle's). */
uint64_t kq_stream_key(uint64_t seed, uint64_t tensor);

/* ---- GGUF model files (host only: no GPU, no context) ---------------------------------------
 * The GGML project's model file format, the on-disk source of k-quant weights (kernite has no
 * file loader; this is the data format on the input side of kq_matvec). A GGUF tensor stores a
 * matrix exactly as kq_matvec takes it: dims[0] = k elements per row, dims[1] = rows, rows back
 * to back; its `type` is the GGML type number, KQ_TYPE_Q4_K / KQ_TYPE_Q6_K for the two this
 * library multiplies. kq_gguf_open maps the file read-only and checks every length in it
 * against the file's size (a malformed file is KQ_E_INVALID with the reason, never a crash);
 * tensor data are read in place, valid until kq_gguf_close. GGUF versions 2 and 3. */
typedef struct kq_gguf kq_gguf;
typedef struct kq_gguf_tensor {
    const char* name;   /* NUL-terminated, owned by the kq_gguf */
    uint32_t type;      /* GGML type number */
    uint32_t n_dims;    /* 1..4 */
    uint64_t dims[4];   /* dims[0] innermost (elements per row); unused ones are 1 */
    uint64_t offset;    /* byte offset of the data in the file */
    uint64_t nbytes;    /* data bytes; 0 when the type's block size is not known to the reader */
    const void* data;   /* host address of the data in the mapping */
} kq_gguf_tensor;
int kq_gguf_open(const char* path, kq_gguf** out);
int kq_gguf_close(kq_gguf* g);
uint64_t kq_gguf_tensor_count(const kq_gguf* g);
int kq_gguf_tensor_at(const kq_gguf* g, uint64_t index, kq_gguf_tensor* out);
int kq_gguf_find(const kq_gguf* g, const char* name, kq_gguf_tensor* out);
/* Metadata: an integer-typed (or bool) value, sign-extended; a string value (owned by g). */
int kq_gguf_meta_int(const kq_gguf* g, const char* key, int64_t* out);
int kq_gguf_meta_str(const kq_gguf* g, const char* key, const char** out);

/* ---- A decode step's attention: rotary embedding, the key/value cache, GQA attention -------
 *
 * Between a layer's q|k|v matvec and its output projection a Llama decode step rotates the query
 * and key heads by their position (RoPE), appends the key and value heads to a cache, and lets
 * each query head attend over every cached position of its key/value head (grouped-query
 * attention: n_heads / n_kv query heads share one). The functional model is kernite's microgpt
 * attention (examples/microgpt/src/gpu.rs:130-230: per head the logits q.k scaled, their maximum,
 * exponentials and sum, the weights and the values they weigh); kernite has no cache, no RoPE and
 * no GQA. Caches are f16, row p = position p, n_kv * head_dim values (head-major); activations
 * are f32. */

/* qkv = the step's q (n_heads * head_dim), k and v (n_kv * head_dim each), back to back, as a
 * q|k|v matvec writes them. q_out <- q with element pairs (2i, 2i+1) of each head rotated by the
 * angle pos * base^(-2i / head_dim) (GGML's "norm" rotary mode; base 10000 for Llama 2, 500000 for
 * Llama 3); row pos of k_cache <- k rotated the same way, row pos of v_cache <- v, as f16. */
int kq_rope_append(kq_ctx* ctx, uint64_t qkv, uint64_t q_out, uint64_t k_cache, uint64_t v_cache,
                   uint32_t n_heads, uint32_t n_kv, uint32_t head_dim, uint32_t pos, double base,
                   kq_stream stream);

/* out[h * head_dim + j] = sum_p w_hp v_p[g(h) * head_dim + j] over the cache's first len rows,
 * w_h = softmax_p(q_h . k_p[g(h)] / sqrt(head_dim)), g(h) = h / (n_heads / n_kv). Split over
 * positions across CTAs, combined in a second launch; workspace (device, 16-byte aligned, not
 * read before written) holds the splits: kq_attention_workspace gives its size. n_heads / n_kv
 * 1..16, head_dim a multiple of 8 up to 256. */
int kq_attention_decode(kq_ctx* ctx, uint64_t out, uint64_t q, uint64_t k_cache, uint64_t v_cache,
                        uint32_t n_heads, uint32_t n_kv, uint32_t head_dim, uint32_t len,
                        uint64_t workspace, uint64_t workspace_bytes, kq_stream stream);
uint64_t kq_attention_workspace(kq_ctx* ctx, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim,
                                uint32_t len);

/* ---- Row-sharded stacks: a matvec whose epilogue also pushes its outputs to other GPUs ----
 *
 * With the rows of a matrix split over N GPUs, every GPU needs the whole output vector for the
 * next matvec. kq_matvec_push does the exchange inside the matvec: each output row r <
 * push_rows is also stored at y[p] + r for every p < npush (the full-vector buffers of all
 * ranks, this one included, mapped with kq_peer_open), and each CTA, once its rows are stored
 * everywhere, adds its row count to counter[p] with a system-scope fence before it. A launch
 * whose x is such a full vector first waits (bounded, acquire) until its rank's counter
 * wait_counter reaches (*epoch - 1) * wait_mul + wait_add, then reads x through L2. Batch 1:
 * the warp-MMA integer kernel (Q4_K, Q5_K, Q6_K; the weights streaming while the wait runs), or
 * the CUDA-core kernel with KQ_FLAG_CUDA_CORES (Q4_K, Q6_K). No reference counterpart: kernite
 * has no collective; its only inter-GPU operation is Buffer::copy_from over cuMemcpyPeer
 * (crates/cuda/src/lib.rs:405-439). */
typedef struct kq_push_desc {
    uint32_t npush;        /* ranks to store to (0..8) */
    uint32_t push_rows;    /* output rows (in output units) that are pushed: rows [0, push_rows) */
    uint64_t y[8];         /* per rank: address of this rank's slice in that rank's full vector */
    uint64_t counter[8];   /* per rank: its arrival counter (u64) for that full vector */
    uint64_t wait_counter; /* 0, or this rank's counter for x (u64) */
    uint64_t epoch;        /* address of this rank's token counter (u64), read on the device */
    uint64_t wait_mul, wait_add;
    /* KQ_PUSH_TAGGED (warp-MMA kernel): full vectors are tagged, 8 bytes an element (the f32
     * value in the low word, a u32 tag in the high word, stored together in one 8-byte store), so
     * a reader needs no counter and no fence: it reads x (when wait_counter is nonzero, or always
     * with KQ_PUSH_TAGGED_X) waiting, bounded, on each element until its tag equals
     * (*epoch - 1) * wait_mul + wait_add (mod 2^32), and the outputs go to y[p] (tagged, element
     * index = output index) with the tag (*epoch - 1) * push_mul + push_add; counter[] unused.
     * Tags of 0 never match (they are what zeroed memory holds): make every tag at least 1. */
    uint32_t flags;
    uint32_t reserved;
    uint64_t push_mul, push_add;
    /* Tagged pushes only. ksplit (0 or 1: none; 2, 4, 8): the CTAs share each row range ksplit
     * ways, each multiplying its share of the row's K-tiles (at most the tiles a row has), and
     * push their partial sums into slot (CTA mod ksplit) of the destination vectors, slots
     * npush * push_rows elements apart (no product epilogue; y is not written). x_slots (0 or 1:
     * none; up to 8): x is such a vector, its slots k elements apart, and every element of x is
     * the sum of its slots, added in slot order. For row-sharded stacks whose shards are too
     * short to give every CTA a row range of its own. */
    uint32_t ksplit, x_slots;
} kq_push_desc;
enum { KQ_PUSH_TAGGED = 1u << 0, KQ_PUSH_TAGGED_X = 1u << 1 };

int kq_matvec_push(kq_ctx* ctx, const kq_matvec_desc* desc, const kq_push_desc* push,
                   kq_stream stream);

/* dst[i] = the value of tagged element i of src (0 <= i < n), once its tag equals
 * (*epoch - 1) * wait_mul + wait_add (mod 2^32): bounded waits, stream-ordered; the last vector of
 * a step (the logits) into plain f32 for the caller. A wait that gives up sets the device error
 * word and the element is copied as it is. */
int kq_tagged_unpack(kq_ctx* ctx, uint64_t dst, uint64_t src, uint64_t n, uint64_t epoch,
                     uint64_t wait_mul, uint64_t wait_add, kq_stream stream);

/* Stream-ordered wait (one thread, bounded, acquire) until *counter >= (*epoch - 1) * wait_mul +
 * wait_add, for a caller that reads a pushed full vector with its own code (the last one of a
 * step, which no later kq_matvec_push waits for). A wait that gives up sets the device error
 * word (kq_device_error) and returns, so the stream goes on. */
int kq_wait_counter(kq_ctx* ctx, uint64_t counter, uint64_t epoch, uint64_t wait_mul,
                    uint64_t wait_add, kq_stream stream);

/* ---- Chains: several matvecs in one launch, with the exchange of a row-sharded stack ---------
 *
 * A decode step is a chain of matvecs, each reading the previous one's output. kq_matvec_chain
 * runs up to 8 of them (batch 1, one type, one k: e.g. a layer's q|k|v, o and gate|up
 * projections) in one launch of the warp-MMA integer kernel, one CTA per SM: each CTA streams its
 * share of the rows of every matrix in turn, the next matrix's weights already in flight while
 * it finishes one. What a kernel boundary did between two matvecs, counters do: once a CTA's
 * outputs of a job are stored, it adds their count to the job's counter (release); a job with a
 * wait_counter reads x only once that counter reaches (*epoch) * wait_target (bounded wait,
 * acquire), i.e. once every CTA (of every rank) has stored its part of x in this step. Counters
 * only grow; *epoch, advanced once per step (kq_epoch_advance), keeps each step's targets apart,
 * so counters and epoch start at zero and are never reset.
 *
 * Row-sharded over N GPUs (one process each): each rank runs the same chain on its rows; a job
 * with npush > 0 also stores its outputs [0, push_rows) into every rank's full vector (push_y[p],
 * this rank's slice in rank p's memory, mapped with kq_peer_open; this rank's own included) and
 * adds the count to counter[p] on each rank (system scope), so the next job's wait on this
 * rank's counter (target N * push_rows per step) is the all-gather. A wait that gives up sets the
 * ctx's device error word and the chain runs on without waiting, so a missing rank costs one
 * wait budget (about 2 s), not a hang. No reference counterpart: kernite launches one kernel at a
 * time and has no collective; its only inter-GPU operation is Buffer::copy_from over
 * cuMemcpyPeer (crates/cuda/src/lib.rs:405-439). */
typedef struct kq_chain_job {
    kq_matvec_desc mv;     /* batch 1; y receives every output of the job on this GPU */
    uint64_t wait_counter; /* 0, or a u64 counter on this GPU that x waits for */
    uint64_t wait_target;  /* the count wait_counter gains per step */
    uint32_t npush;        /* 0, or the ranks (<= 8) whose full vectors receive pushed outputs */
    uint32_t push_rows;    /* outputs [0, push_rows) are pushed */
    uint64_t push_y[8];    /* per rank: where this rank's pushed outputs go in that rank's memory */
    uint64_t counter[8];   /* npush == 0: counter[0] (0 = none) on this GPU gains the output
                            * count; npush > 0: counter[p] on rank p gains the pushed count */
} kq_chain_job;

/* Runs jobs[0..njobs) (1..8) in one launch on `stream`; epoch is the address of this GPU's u64
 * step counter. Every job has the first one's type (Q4_K, Q5_K or Q6_K) and k and must fit the
 * integer kernel's shared memory (KQ_E_UNSUPPORTED otherwise). The first job also waits for the
 * previous kernel on the stream, as every matvec does. */
int kq_matvec_chain(kq_ctx* ctx, const kq_chain_job* jobs, uint32_t njobs, uint64_t epoch,
                    kq_stream stream);

/* *epoch += 1 on `stream` (one thread): the start of a step for the chains that follow. */
int kq_epoch_advance(kq_ctx* ctx, uint64_t epoch, kq_stream stream);

/* Device memory other GPUs can map: cudaMalloc'd, zeroed, with its CUDA IPC handle (64 bytes)
 * written to ipc_handle. Replaces the peer side of Buffer::copy_from (crates/cuda/src/lib.rs:
 * 405-439), which copies through cuMemcpyPeer instead of mapping. */
int kq_peer_alloc(kq_ctx* ctx, uint64_t bytes, uint64_t* ptr, void* ipc_handle);
/* Maps another process's kq_peer_alloc memory from its IPC handle (peer access enabled). */
int kq_peer_open(kq_ctx* ctx, const void* ipc_handle, uint64_t* ptr);
/* Unmaps memory kq_peer_open mapped / frees memory kq_peer_alloc allocated. */
int kq_peer_close(kq_ctx* ctx, uint64_t ptr);
int kq_peer_free(kq_ctx* ctx, uint64_t ptr);

/* ---- The kernels as a module image, for a caller that loads and launches them itself -------
 *
 * kernite loads a module (Module::load, crates/cuda/src/lib.rs:945-1016, which takes PTX text only,
 * :952-953) and launches its functions with cuLaunchKernel from a macro launcher
 * (crates/macros/src/gpu.rs:276-328, crates/cuda/src/lib.rs:1045-1054). The pair below lets it do
 * the same with this library's warp-MMA kernels: kq_module_image hands over the sm_100a cubin
 * (tcgen05 and the other sm_100a-only instructions need the architecture-specific target, so the
 * image is a cubin, not PTX; a Module::load_image(&Cuda, &[u8], names) addition to kernite-cuda
 * loads it), and kq_matvec_plan says which function of it to launch, and how. */

/* The image: ELF bytes inside libkq.so, valid for the life of the process. No GPU needed. */
int kq_module_image(const void** image, size_t* bytes);

/* One planned launch of a function of that image. */
typedef struct kq_launch {
    char kernel[256];      /* its name in the image (cuModuleGetFunction) */
    uint32_t grid[3];
    uint32_t block[3];
    uint32_t shared_bytes; /* dynamic shared memory; set the function's
                            * CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES to at least this */
    uint32_t param_bytes;  /* the function takes one parameter: these bytes, by value */
    uint8_t params[512];
} kq_launch;

/* Plans kq_matvec(ctx, desc) on the warp-MMA kernel without launching anything: the function,
 * the grid, the block, the shared memory and the parameter bytes. Launched with
 * cuLaunchKernel(f, grid, block, shared_bytes, stream, {params}, NULL) in the primary context of
 * the ctx's GPU (the one kernite retains), it computes what kq_matvec computes, bit for bit; its
 * bounded waits record into the ctx's device error word (kq_device_error). Requests the warp-MMA
 * kernel does not serve (batch above 8, tensor-core or CUDA-core flags) are KQ_E_UNSUPPORTED. */
int kq_matvec_plan(kq_ctx* ctx, const kq_matvec_desc* desc, kq_launch* out);

/* The tensor-core Q4_K matvec of kq_matvec_q4k (batch 1..64) for callers that cannot allocate
 * device memory: code running while a CUDA graph is being captured, a serving process whose
 * memory pool has already reserved the GPU, or a latency-critical path where a cudaMalloc
 * would stall. It takes no kq_ctx (creating one allocates) and calls no cudaMalloc, cudaFree
 * or other allocating routine. No counterpart in the reference: kernite always allocates
 * through Cuda::alloc.
 *   - Its scratch (X in f16, k * npad * 2 bytes, npad = batch rounded up to 16, 32 or 64) is a
 *     static 1 MiB device array that every GPU loading the library holds until the process
 *     exits; larger requests (k > 32768 up to batch 16, > 16384 up to 32, > 8192 up to 64) are
 *     rejected with KQ_E_INVALID and a message saying so.
 *   - All calls share that array and it keeps the last call's contents; each call rewrites all
 *     of it that it reads. Calls that overlap on the GPU (different streams, or different host
 *     threads) race on it: serialise them.
 *   - The first call on a device sets that device up (attributes, kernel limits, the array's
 *     device address) with the device current; make it before any stream capture.
 * y is batch x rows f32 (row stride rows), x is batch x k f32 (stride k), W as kq_matvec_q4k. */
int kq_matvec_q4k_noalloc(uint64_t y, uint64_t w, uint64_t x, uint32_t rows, uint32_t k,
                          uint32_t batch, kq_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* KQ_H */
