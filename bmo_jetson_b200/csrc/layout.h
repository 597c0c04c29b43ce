// layout.h -- HBM layouts and kernel argument blocks shared by host and device.
//
// Q4_0 weights are repacked at load time from ggml's row-major 18-byte blocks
// (fp16 d + 16 bytes of nibbles) into "row tiles": 32 rows x all blocks,
// cut into chunks of 8 blocks.  One chunk is 4608 contiguous bytes:
//   [8 blocks][32 rows][16 B nibbles]  (4096 B, row r's block at blk*512 + r*16)
//   [8 blocks][32 rows][fp16 d]        (512 B)
// so a warp reads one block of 32 rows as a single 512-byte coalesced line,
// the activation block is a shared-memory broadcast, and every chunk is a
// 16-byte aligned bulk copy.  The bytes per weight are unchanged (18 per 32).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define BMO_HD __host__ __device__
#else
#define BMO_HD
#endif

namespace bmo {

constexpr int kTileRows = 32;
constexpr int kChunkBlocks = 8;
constexpr int kChunkQsBytes = kChunkBlocks * kTileRows * 16;   // 4096
constexpr int kChunkBytes = kChunkQsBytes + kChunkBlocks * kTileRows * 2;  // 4608

// The chunks of one row tile in the reference GEMV's chain order.  The
// reference (bmo_cuda_kernels.cu:560-683) gives lane l = 2m + h of a row's
// warp half block h of the blocks m (mod 16); its accumulator j chains blocks
// 64 i + 16 j + m, and blocks past the last whole group of 64 (the tail, in
// steps of 16) continue accumulator 0.  A chunk's 8 blocks therefore share one
// key group G = 2 j + m / 8: main chunk c (tile-local) has G = c % 8 and chain
// position c / 8, tail chunk nm + t has G = t % 2 and position nmg + t / 2.
struct KeyChains {
    int nm;     // main chunks per tile: 8 * (blocks / 64)
    int nmg;    // main chunks per key group
    int ntail;  // tail chunks per tile (the last may hold padding blocks)
    BMO_HD static KeyChains of(int nb, int cpt) {
        KeyChains k;
        k.nmg = nb / 64;
        k.nm = 8 * k.nmg;
        k.ntail = cpt - k.nm;
        return k;
    }
    // chunks of key group g, and the tile-local index of its p-th chunk
    BMO_HD int len(int g) const { return nmg + ((g < 2 && ntail > g) ? (ntail - g + 1) / 2 : 0); }
    BMO_HD int chunk(int g, int p) const { return p < nmg ? g + 8 * p : nm + g + 2 * (p - nmg); }
    // key groups that hold chunks (the others contribute +0 to every lane)
    BMO_HD int groups() const { return nmg > 0 ? 8 : (ntail < 2 ? ntail : 2); }
};

// Row order inside a tile.
enum RowPerm : int {
    kPermIdentity = 0,  // lane l of tile t is row 32t + l
    kPermSwiGLU = 1,    // lanes 0-15 gate rows 16t+l, lanes 16-31 up rows F+16t+l-16
};

// Prologue: how the GEMV input vector reaches shared memory as Q8_1 blocks.
enum Prologue : int {
    kProPlain = 0,    // quantise fp32 x
    kProNorm = 1,     // RMSNorm(x) * gamma, then quantise
};

// Epilogue: what happens to the finished dot products of a tile.
enum Epilogue : int {
    kEpiStore = 0,   // y = acc (+ bias)
    kEpiResid = 1,   // y = resid + acc
    kEpiSwiGLU = 2,  // act = silu(gate) * up
    kEpiQKV = 3,     // RoPE on q/k, append k/v into the ring cache, q out
    kEpiLogits = 4,  // logits (+ bias) and per-tile (max, argmax)
    kEpiEmbAdd = 5,  // y = acc + embedding row of a token
    kEpiPartial = 6, // ypart = acc in double, unrounded (tensor-parallel partial sums)
};

enum KvType : int { kKvF16 = 0, kKvQ4_0 = 1 };

// ggml tensor element types used by embedding tables.
enum GgmlType : int { kTF32 = 0, kTF16 = 1, kTQ4_0 = 2, kTQ8_0 = 8, kTI32 = 26, kTBF16 = 30 };

struct QMatDesc {
    const uint8_t *tiles;  // device, n_tiles * cpt * kChunkBytes
    int rows;              // logical rows
    int cols;              // logical cols (multiple of 32)
    int nbx;               // blocks per row incl. padding (multiple of 8)
    int cpt;               // chunks per tile = nbx / 8
    int n_tiles;
    int perm;
    int swiglu_f;          // F for kPermSwiGLU
};

// Source of a token id for an embedding lookup: either a device int, or the
// reduction of per-tile (max, argmax) pairs left by a logits epilogue.
struct TokenSrc {
    const int *tok;        // used when pairs == nullptr
    const float2 *pairs;   // (value, index-as-float bits) per tile
    int n_pairs;
    int *tok_out;          // optional: resolved token written here (one thread)
};

struct EmbTable {
    const void *data;
    int type;              // GgmlType
    int rows;              // vocabulary rows
    int dim;               // row length
    long long row_bytes;
};

struct AttnArgs {
    const float *q;          // [n_heads][hd] rotated queries
    const float *v_raw;      // [n_kv][hd] fp32 v of this token
    const void *k_cache, *v_cache;
    const uint8_t *k_scale, *v_scale;
    long long kv_layer_off;  // element offset of this layer
    int n_heads, n_kv_heads, n_ctx, kv_type;
    const int *pos;
    float scale;
    float *out;              // [n_heads][hd]
    int *status;
    // batched sessions (grid z): row s reads q/v_raw/out at + s * qo_stride
    // (vraw_stride), its position at pos[s * pos_stride], and the ring of
    // session ring_of[s] (s when null) at + ring * kv_sess_stride elements
    long long kv_sess_stride;
    int qo_stride, vraw_stride, pos_stride;
    const int *ring_of;
};

struct GemvArgs {
    QMatDesc W;
    // prologue
    const float *x;
    const float *gamma;
    float eps;
    float *xn_out;         // optional: CTA 0 writes the normalised vector
    uint8_t *q8_out;       // optional: CTA 0 writes the Q8_1 blocks (36 B each)
    // epilogue
    float *y;
    const float *resid;
    const float *bias;
    float2 *argmax_pairs;
    int argmax_limit;      // rows >= limit excluded from the argmax
    // qkv epilogue
    int q_dim, kv_dim, head_dim;
    const float2 *rope_cs; // [head_dim/2] (cos, sin) for this position, or null (no RoPE)
    void *k_cache, *v_cache;        // fp16 or Q4_0 planes
    uint8_t *k_scale, *v_scale;     // Q4_0 fp16 scale planes
    int kv_type, n_ctx;
    const int *pos;        // device position (slot = pos % n_ctx)
    long long kv_layer_off;  // element offset of this layer in the cache planes
    float *v_out;          // raw fp32 v (window-of-one case)
    // embedding-add epilogue
    EmbTable emb;
    TokenSrc tok;
    // partial-sum epilogue: [rows] doubles
    double *ypart;
    // work split: tile_aligned = 1 gives every CTA whole row tiles (no
    // cross-CTA combine); 0 splits the (tile, chunk) units evenly (stream-K)
    int tile_aligned;
    // stream-K bookkeeping
    double *gpart;         // [n_tiles][cpt+1][32] per-owner partial sums
    int *gcount;           // [n_tiles], zero between launches
    int *status;
};


// One step of a decode frame.  The engine builds a frame as a list of these
// and launches one kernel per entry.
enum PhaseKind : int {
    kPhGemv = 0,      // g with prologue `pro`, epilogue `epi`
    kPhAttn = 1,      // decode attention `at` (head_dim, `splits` CTAs per head in the per-op path)
    kPhTokenOut = 2,  // CTA 0 writes the first maximum over tok.pairs into tok.tok_out
    kPhAllReduce = 3, // tensor parallel: sum g.ypart[0..count) over the ranks (double, in place)
    kPhResidAdd = 4,  // tensor parallel: g.y[i] = g.resid[i] + (float)g.ypart[i], i < count
    kPhTpExchange = 5,  // tensor parallel over peer memory: g.y[i] = g.resid[i] + (float)(sum over ranks r,
                        // in rank order, of rank r's partial buffer `splits`)[i], i < count
};

// ---- tensor parallel exchange over peer memory ----
// Every rank owns one exchange block (cudaMalloc, mapped into the other ranks
// through CUDA IPC): two partial-sum buffers of kTpBufDoubles doubles (the
// split projections of a layer alternate between them), then one 64-bit
// arrival word per source rank.  A rank signals "my buffer is complete for
// exchange e" by storing e into its word of every peer's block (release, system
// scope); a rank sums the buffers once every peer's word in its own block
// has reached e.  kTpBlockBytes covers both buffers and the words.
constexpr int kTpMaxRanks = 8;
constexpr int kTpBufDoubles = 8192;
constexpr size_t kTpFlagOffset = 2 * kTpBufDoubles * sizeof(double);
constexpr size_t kTpBlockBytes = kTpFlagOffset + kTpMaxRanks * sizeof(unsigned long long) + 64;
struct TpExchangeArgs {
    const double *part[kTpMaxRanks];           // rank r's partial buffer of this exchange (peer memory for r != rank)
    unsigned long long *flag_out[kTpMaxRanks];  // this rank's arrival word in rank r's block
    const unsigned long long *flag_in;          // this rank's arrival words, one per source rank
    unsigned long long *seq;                    // exchanges this rank has completed (device counter)
    const float *resid;
    float *y;
    int *status;
    int rank, size, n;
};

struct FramePhase {
    int kind;
    int pro, epi;
    int head_dim;
    int splits;
    GemvArgs g;
    AttnArgs at;   // kPhAttn
    TokenSrc tok;  // kPhTokenOut
    int count;     // kPhAllReduce, kPhResidAdd
};

// ---- the depformer cascade as one launch on one thread-block cluster ----
// One entry per weight matrix in execution order: per codebook step, the
// input projection, then per layer QKV, O, FFN-in and FFN-out, then the head.
enum DepOpKind : int { kDepIn = 0, kDepQKV = 1, kDepO = 2, kDepFfnIn = 3, kDepFfnOut = 4, kDepHead = 5 };
constexpr int kDepMaxSteps = 8;
struct DepOp {
    QMatDesc W;
    const float *gamma;        // RMSNorm weight of the input (QKV, FFN-in), else null
    const float *gamma_ahead;  // the RMSNorm weight two normalised ops later (prefetched into this one's buffer)
    int kind;                  // DepOpKind
    int layer, step;
    int norm_idx;              // ordinal among the normalised ops (selects the weight buffer and its phase)
};
struct DepCascadeArgs {
    const DepOp *ops;          // device table of n_ops entries
    int n_ops;
    const float *gamma0[2];    // RMSNorm weights of the first two normalised ops
    EmbTable emb[kDepMaxSteps];  // token table of step cb's input (cb 0: the text-token table)
    const float *z;            // [n_embd] the temporal transformer's normalised output
    int n_embd;
    TokenSrc first;            // step 0's input token (the text token)
    int *tok_out;              // [1 + dep_q]: the text token, then each step's argmax
    float *logits;             // [dep_q][logits_stride]
    int logits_stride;
    float2 *pairs;             // optional [dep_q][pairs_stride] per-tile (max, argmax)
    int pairs_stride;
    __half *k_cache, *v_cache; // [n_layers][heads][n_ctx][hd] fp16 (written for the per-step API)
    int dep_q, n_layers, dim, ffn, heads, hd, n_ctx, argmax_limit;
    float eps, scale;
    int *status;
    // grid-wide variant: two exchange buffers of ll_stride 64-bit words
    // (epoch << 32 | value bits) and the launch counter that makes epochs unique
    unsigned long long *ll;
    int ll_stride;
    unsigned int *seq;
};

// ---- the caller's frame loop on the device (bmo_daemon.cpp:641-816) ----
// The daemon's per-frame state: the tokens fed back into the next frame, the
// std::mt19937 its samplers share, and this frame's results.
constexpr int kLoopCb = 8;          // audio codebooks of an agent (and of the user)
constexpr int kLoopTopKMax = 2048;  // largest top-k the device sampler takes (the audio vocabulary)
constexpr int kSampleMaxN = 32768;  // most logits the device sampler draws from (Moshi text: 32000)
constexpr int kLoopOut = 1 + 2 * kLoopCb;  // a frame's results: text, audio[8], codec input[8]
constexpr int kLoopRing = 64;       // frames of results kept on the device
// The caller's per-frame inputs, copied to the device before each frame.
struct LoopParams {
    int sampling;               // 0: greedy everywhere (the daemon without --sampling)
    float temp_text, temp_audio;
    int top_k_text, top_k_audio;
    int user_valid;             // 0: the daemon's silence tokens stand for the user
    int user[kLoopCb];          // the user's audio tokens of this frame
};
struct LoopState {
    LoopParams in[kLoopRing];   // frame f's inputs in row f % kLoopRing
    int frame;                  // frames decoded so far (the temporal position)
    int prev_text;              // the text channel's token for the next frame
    int prev_audio[kLoopCb];    // the agent's audio tokens of the last frame
    int prev_user[kLoopCb];     // the user's audio tokens of the last frame
    int prev_cb0;               // the agent's codebook-0 token of the last frame
    int user[kLoopCb];          // this frame's user tokens
    int next_text;              // this frame's text token
    int audio[kLoopCb];         // this frame's audio tokens
    int mti;                    // std::mt19937 position
    unsigned mt[624];           // std::mt19937 state
    int out[kLoopRing][kLoopOut];  // frame f's results in row f % kLoopRing
};
// Fixed by the model.
struct LoopConfig {
    int text_n, audio_n;        // logits the samplers consider (32000, 2048 for Moshi)
    int text_pad, audio_pad;    // the channels' "no token yet" ids (32000, 2048)
    int n_tok;                  // input channels: 1 + 8 agent (+ 8 user when 17)
};
// One draw from logits[0, n): the text draw (`text` != 0) stays greedy when
// the first argmax is a pause token (3 or 0).  Its parameters are the frame
// loop's (st->in[st->frame % kLoopRing]) when st is set, else the fields
// here; mt[624] and *mti are the std::mt19937 state it advances.
struct SampleArgs {
    const float *logits;
    int n, text;
    const LoopState *st;
    int sampling, top_k;
    float temp;
    unsigned *mt;
    int *mti;
    int *out;
};

// ---- batched sessions (config 4) ----
// Q8_1 activations of S sessions, block-major, padded to P = S rounded up to
// 16 sessions, laid out as the tensor core's B operand with the two half
// blocks of the reference's dot product (packed bytes 0-7 of a Q4_0 row hold
// elements 0-7 and 16-23, bytes 8-15 elements 8-15 and 24-31) on separate
// rows: block b occupies 64 P bytes at xq + b * 64 P; row R = 2s carries
// session s's codes 0-7 and 16-23, row 2s + 1 its codes 8-15 and 24-31, each
// at its own element position with zeros elsewhere, in the K-major canonical
// layout of 8-row x 16-byte core matrices: bytes [16k, 16k + 16) of row R at
// (R / 8) * 256 + k * 128 + (R % 8) * 16.  One MMA over the block then yields
// both half-block sums of every session.  The block's scales are 3 P floats
// at xds + 3 P b: P / 2 float4 {d8[2p], d8[2p+1], -M d8[2p], -M d8[2p+1]}
// (M = 1.5 * 2^23), then P / 2 float2 {-4 s8[2p], -4 s8[2p+1]}.  The 8 blocks of
// chunk kc are one contiguous run of 512 P bytes (and 96 P bytes of scales).
constexpr int kBatchMax = 64;  // sessions per launch
BMO_HD constexpr int batch_pad(int n_sess) { return (n_sess + 15) & ~15; }
constexpr int kBatchMaxTokens = 64;

// Per-call inputs of a batched frame (one host->device copy): row s runs
// session sess[s] at position pos[s] on tokens[s * kBatchMaxTokens + 0..n_tok).
struct BatchIn {
    int32_t sess[kBatchMax];
    int32_t pos[kBatchMax];
    int32_t tokens[kBatchMax * kBatchMaxTokens];
    int32_t n_tok;
    int32_t pad[3];
};

struct BatchStageArgs {
    const float *x;          // [S][x_stride]
    int x_stride, cols, nbx, n_sess;
    const float *gamma;      // RMSNorm weight, or null (plain)
    float eps;
    float *xn_out;           // optional [S][cols]: the normalised vectors
    int xn_stride;
    int8_t *xq;
    float *xds;
    // optional token lookup for an embedding-add GEMV: session s's token is the
    // first maximum of pairs[s * pairs_stride + 0..n_pairs), or tok_in[s]
    const float2 *pairs;
    int pairs_stride, n_pairs;
    const int *tok_in;
    int *tok;                // [S] resolved tokens
    int *tok_out;            // optional: tok_out[s * tok_out_stride]
    int tok_out_stride;
};

struct BatchGemmArgs {
    QMatDesc W;
    int n_sess;
    const int8_t *xq;
    const float *xds;
    float *y;                // [S][y_stride]
    int y_stride;
    const float *resid;      // [S][resid_stride]
    int resid_stride;
    const float *bias;
    float2 *pairs;           // logits: per-tile (max, argmax) at pairs[s * pairs_stride + t]
    int pairs_stride, argmax_limit;
    // qkv epilogue
    int q_dim, kv_dim, head_dim;
    const float2 *rope;      // [S][head_dim / 2] or null
    void *k_cache, *v_cache;
    uint8_t *k_scale, *v_scale;
    long long kv_sess_stride, kv_layer_off;
    int kv_type, n_ctx;
    const int *pos;          // position of row s at pos[s * pos_stride]
    int pos_stride;
    const int *ring_of;      // KV ring of row s: ring_of[s] (s when null)
    float *v_out;            // raw v [S][v_out_stride]
    int v_out_stride;
    // embedding-add epilogue
    EmbTable emb;
    const int *tok;          // [S]
    int *status;
    // tensor-core path: split row blocks combine through ws (partial sums,
    // one double per (session, row): [row block][contributor][P][128]) and
    // cnt (one zeroed counter per 128-row block)
    float *ws;
    int *cnt;
    int max_contrib;
};

}  // namespace bmo
