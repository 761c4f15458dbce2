// Host/device ABI of the B200 expert-parallel runtime: peer tables, control-block layout, error
// codes and buffer layouts. Every struct here is passed to kernels by value or stored in device or
// host-mapped memory, so sizes are pinned with static_asserts (the same discipline as the
// reference's `CxiGpuContext`/`CxiWindow` ABI header, backend/include/cxi_gin_abi.h:6-60).
#pragma once

#include <cstdint>

namespace ep {

constexpr int kMaxRanks = 8;        // one NVLink/NVSwitch domain (one B200 box)
constexpr int kMaxTopk = 16;
constexpr int kMaxLocalExperts = 1024;
constexpr int kMaxCountCtas = 128;     // CTAs of the dispatch count kernel (per-CTA counts live in the control block)
constexpr int kMaxStageChunks = 256;   // staged-chunk flags per source rank (chunk size >= capacity / 256)
constexpr int kAbiVersion = 2;

// ------------------------------------------------------------------------------------------------
// Error codes written into the host-mapped `ErrorState` by kernels whose bounded waits expire.
// ------------------------------------------------------------------------------------------------
enum ErrorCode : int {
    kOk = 0,
    kErrTimeoutNotify = 1,         // dispatch count step: a peer's counts (or a count CTA's prefix) never arrived
    kErrTimeoutPullDone = 2,       // staging reuse: a receiver never finished pulling the last dispatch
    kErrTimeoutCombineReady = 3,   // combine: destination never finished its previous combine
    kErrTimeoutCombineArrive = 4,  // combine: contributions never all arrived
    kErrTimeoutBarrier = 5,
    kErrTimeoutLLDispatch = 6,
    kErrTimeoutLLCombine = 7,
    kErrTimeoutTma = 8,            // a TMA bulk copy never completed
    kErrTimeoutStaged = 9,         // dispatch pull: a source never staged the chunk holding a wanted token
    kErrCapacity = 10,             // receive capacity exceeded (tokens beyond the buffer)
    kErrBounds = 11,               // an index outside its window (bounds check on every peer store)
    kErrBadArgs = 12,
    kErrTimeoutPP = 13,
    kErrTimeoutAgrs = 14,          // AGRS: a peer never signalled its all-gather copies / session end
    kErrTimeoutTest = 20,          // transport self-test wait expired (used by the delayed-peer test)
};

struct ErrorState {
    int code;
    int peer;
    int detail;
    int rank;
    int reserved[4];
};
static_assert(sizeof(ErrorState) == 32, "ErrorState ABI");

// ------------------------------------------------------------------------------------------------
// Device trace ring: kernels append [start, end, event, block, smid, rank, a, b] records read from
// %globaltimer when `KernelStatus::trace` is non-null (a runtime switch, no rebuild). Records are
// appended with one atomic; a full ring drops records and the host sees `cursor > capacity`.
// ------------------------------------------------------------------------------------------------
enum TraceEvent : int {
    kTraceStage = 100,          // dispatch stage (quantize + records; stage warps or stage block), a = tokens
    kTraceWaitReceivers = 101,  // dispatch: wait for the receivers of the previous dispatch
    kTraceCount = 102,          // dispatch count kernel (lists + count exchange), a = 1 in cached mode
    kTraceCountExchange = 103,  // count kernel: count exchange wait, a = epoch
    kTracePull = 104,           // pull block, a = received tokens
    kTraceCombine = 110,        // combine block (push + reduce), a = 1 for push blocks
    kTraceCombinePush = 111,    // combine push warp finished its rows, a = warp
    kTraceLLDispatchSend = 120,
    kTraceLLDispatchRecv = 121,
    kTraceLLCombineSend = 122,
    kTraceLLCombineRecv = 123,
    kTraceLLDispatchRecvGemm = 124,  // fused receive of the masked GEMM: wait for the peers, a = 1 if complete
    kTraceBarrier = 130,
    kTracePP = 140,             // pipeline copy CTA, a = is_send, b = bytes
};

struct TraceRecord {
    uint64_t start_ns;
    uint64_t end_ns;
    int32_t event;
    int32_t block;
    int32_t smid;
    int32_t rank;
    int32_t a;
    int32_t b;
};
static_assert(sizeof(TraceRecord) == 40, "TraceRecord ABI");

struct TraceRing {
    TraceRecord* records;
    unsigned long long* cursor;
    uint64_t capacity;
};

// Passed by value to every kernel that waits.
struct KernelStatus {
    ErrorState* host_error;  // host-mapped (cudaHostAllocMapped) device pointer
    int* abort_flag;         // device memory; set by the first failing block
    uint64_t timeout_ns;     // wait limit in nanoseconds of %globaltimer
    int rank;
    int pad;
    TraceRing* trace;        // device trace ring, or null (tracing off)
};
static_assert(sizeof(KernelStatus) == 40, "KernelStatus ABI");

// Peer table: base address of the same symmetric region on every rank (index = rank). Entry
// `rank` is the local base. Passed by value (64 bytes).
struct PeerTable {
    void* base[kMaxRanks];
};
static_assert(sizeof(PeerTable) == 64, "PeerTable ABI");

// ------------------------------------------------------------------------------------------------
// Control block at offset 0 of the normal-mode (NVL) region. Every flag is written by the party
// that signals and read by the party that waits in ITS OWN memory (signals are pushed, never
// polled across NVLink). All epochs are monotonically increasing call sequence numbers.
// ------------------------------------------------------------------------------------------------
struct alignas(128) NormalCtrl {
    int notify_flag[kMaxRanks];             // [src] = dispatch epoch once src's counts/list/staging are ready
    int pull_done[kMaxRanks];               // [dst] = dispatch epoch once dst finished reading my staging
    int combine_ready[kMaxRanks];           // [dst] = combine seq once dst finished reducing (its slots are free)
    int barrier_flag[kMaxRanks];            // [src] = barrier epoch
    int combine_arrived;                    // rows of combine contributions that landed here (reset by reducer)
    int combine_reduced_blocks;             // reducer blocks that finished (reset by the last one)
    int pull_finished_blocks;               // pull blocks that finished (reset by the last one)
    // Device-resident sequence numbers (local to this rank). Kernels read and advance them, so no
    // per-call value is baked into a launch and captured CUDA graphs replay correctly.
    int dispatch_epoch;                     // last dispatch whose notify completed
    int combine_seq;                        // last combine whose reduce completed
    int barrier_epoch;                      // last barrier
    int combine_token_cursor;               // next token for the combine reducers (reset by the last block)
    int pad0[25];
    int token_counts[2][kMaxRanks][kMaxRanks];  // [parity][src][dst] tokens src sends to dst
    int expert_counts[2][kMaxRanks][kMaxLocalExperts];  // [parity][src][local expert] tokens from src
    // Overlapped stage: the source's stage warps release staged[src][chunk] = dispatch epoch in every
    // receiver's block once all tokens of that chunk are in its staging; pull producers wait on it.
    int staged[kMaxRanks][kMaxStageChunks];
    int stage_chunk_done[kMaxStageChunks];      // local: tokens of each chunk staged so far (reset by count)
    // Count kernel (local): per-CTA per-destination token counts, published with the epoch in
    // count_cta_flag so that later CTAs add up their predecessors' counts (ordered lists).
    int count_cta_flag[kMaxCountCtas];
    int count_cta_counts[kMaxCountCtas][kMaxRanks];
    int count_done_ctas;                        // local ticket; the last CTA exchanges counts (and resets it)
    int selftest_flag;                          // transport self-test: peers add to it, the owner waits
    int probe_flag;                             // NVLink micro-probe: flag round trips (peer writes, owner waits)
    int pad1[29];
};
static_assert(sizeof(NormalCtrl) % 128 == 0, "NormalCtrl alignment");

// Host-mapped per-buffer workspace read by the CPU after the notify step (the reference's
// `moe_recv_counter` / `moe_recv_expert_counter`, [DE]csrc/legacy/buffer.hpp:579-597).
struct HostCounters {
    int ready_ticket;              // = host ticket of the dispatch whose fields below are valid
    int num_recv_tokens;
    int num_local_experts;
    int pad;
    int num_recv_tokens_per_expert[kMaxLocalExperts];
};

// ------------------------------------------------------------------------------------------------
// Normal-mode region layout (a pure function of region size, hidden, top-k and ranks, so every rank
// computes the same offsets). Offsets are relative to the region base.
// ------------------------------------------------------------------------------------------------
struct NormalLayout {
    int64_t ctrl_off;
    int64_t list_off;        // int32 [kMaxRanks][capacity]: token ids I send to each destination
    int64_t staging_off;     // records [capacity], record_bytes each
    int64_t combine_off;     // bf16 rows [capacity * num_ranks][hidden]
    int64_t combine_w_off;   // f32 [capacity * num_ranks][topk_pad]
    int64_t scratch_off;     // local only: [capacity] spare bytes, then int32 per-expert token counters [kMaxExperts] (zero between calls)
    int64_t arrival_off;     // int32 [capacity]: combine contributions landed per token (peers add, reducer resets)
    int64_t total_bytes;
    int32_t capacity;        // max tokens per rank per call
    int32_t hidden;
    int32_t num_topk;
    int32_t topk_pad;        // top-k rounded up to a multiple of 4 (16-byte metadata)
    int32_t record_bytes;    // staging record stride
    int32_t num_ranks;
};
static_assert(sizeof(NormalLayout) == 88, "NormalLayout ABI");
constexpr int kMaxExperts = kMaxRanks * kMaxLocalExperts;

// Staging record of one token (written by its source rank, pulled by receivers):
//   [x: hidden * elem bytes][scales: f32 * hidden/128 (fp8 only)][topk_idx: i32 * topk_pad][topk_w: f32 * topk_pad]
struct RecordFormat {
    int32_t x_bytes;
    int32_t scale_off;
    int32_t scale_bytes;
    int32_t idx_off;
    int32_t w_off;
    int32_t bytes;  // total, 16-byte multiple
};

// ------------------------------------------------------------------------------------------------
// Low-latency region layout: two halves (double buffering, at most two live results, the
// reference's rule at [DE]deep_ep/buffers/legacy.py:425-426).
// ------------------------------------------------------------------------------------------------
struct LLLayout {
    int64_t half_bytes;
    // offsets relative to a half base
    int64_t ctrl_off;           // LLCtrl
    int64_t recv_x_off;         // [E_l][R*maxT][hidden] (bf16 capacity; fp8 uses hidden bytes per row)
    int64_t recv_scales_off;    // f32 [E_l][hidden/128][R*maxT] (column-major per expert)
    int64_t recv_src_info_off;  // i32 [E_l][R*maxT] source token index
    int64_t recv_src_meta_off;  // i32 [E_l][R*maxT] src_rank * topk + k
    int64_t combine_recv_off;   // bf16 [maxT][topk][hidden]
    int64_t combine_send_off;   // bf16 [E_l][R*maxT][hidden] zero-copy send buffer
    int64_t combine_meta_off;   // u32 [maxT][topk][hidden/128] LogFMT group metadata (amax | amin << 16)
    int32_t max_tokens;
    int32_t hidden;
    int32_t num_experts;
    int32_t num_local_experts;
    int32_t num_ranks;
    int32_t num_topk;
};

// LL flags are set to 1 by the sender and reset to 0 by the receiver once every receive block has
// seen them (no sequence numbers, so captured CUDA graphs replay). A half is reused two calls later,
// after the alternation of dispatch/combine has ordered the receiver's reset before the next write.
struct alignas(128) LLCtrl {
    int dispatch_done[kMaxRanks];   // [src] = 1 once src's messages to me all landed
    int combine_done[kMaxRanks];    // [src] = 1 once src's rows to me all landed
    int send_finished_blocks;       // local: blocks that finished the send phase (reset by last)
    int csend_finished_blocks;
    int recv_finished_blocks;       // local: dispatch receive blocks that saw every flag
    int crecv_finished_blocks;
    int pad[12];
    int slot_counter[kMaxLocalExperts];  // [local expert] slots claimed by senders (remote atomics)
};

// ------------------------------------------------------------------------------------------------
// Symmetric side region (pipeline send/recv, AGRS sessions, Engram storage): one CUDA-IPC region per
// feature and rank, [SymCtrl | data]. Every flag here is written by the PEER named in its comment
// and waited on locally (signals live in the waiter's memory).
// ------------------------------------------------------------------------------------------------
constexpr int kMaxAgrsSlots = 64;            // all-gathers per AGRS session
constexpr int64_t kSymCtrlBytes = 64 * 1024; // data starts here (TMA / vector aligned)

struct alignas(128) SymCtrl {
    // Pipeline ring. Direction d = 0: the neighbour is my PREV rank (it sends with dst == its next);
    // d = 1: the neighbour is my NEXT rank. With two ranks both neighbours are one rank and d = 0.
    int pp_arrival[2];      // written by neighbour d: tensors it has delivered into my slot set d
    int pp_release[2];      // written by neighbour d: tensors of mine it has consumed
    int pp_send_count[2];   // local: tensors sent towards neighbour d
    int pp_recv_count[2];   // local: tensors received from slot set d
    int pp_send_ticket[2];  // local CTA tickets (last CTA signals)
    int pp_recv_ticket[2];
    int pad0[20];
    int barrier_signal[kMaxRanks];                    // written by peer r: barrier epoch
    int agrs_session_signal[kMaxRanks];               // written by peer r: AGRS session it finished
    int agrs_recv_signal[kMaxAgrsSlots][kMaxRanks];   // written by peer r: its copy of slot s arrived (value = session)
    // Down projection with the combine send as its epilogue (one region per layer, epochs from the host).
    int gc_done[kMaxRanks];   // written by peer r: last epoch whose rows r stored into my slots
    int gc_free[kMaxRanks];   // written by peer r: last epoch r finished reducing (its slots are free)
    int gc_send_blocks;       // local: GEMM CTAs that finished the send (reset by the last one)
    int gc_reduce_blocks;     // local: reduce blocks that finished (reset by the last one)
};
static_assert(sizeof(SymCtrl) <= kSymCtrlBytes, "SymCtrl must fit in the control block");

}  // namespace ep
