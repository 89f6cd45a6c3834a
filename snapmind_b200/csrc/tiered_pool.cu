// Batched tiered KV pool: device-side residency, LRU eviction and
// sink + window pinning (sm_100a).
//
// A fixed pool of chunk slots (one block of `chunk` tokens per slot, all
// layers) holds the resident chunks of many sequences; every chunk also lives
// in host-pinned backing.  Per decode step:
//   1. the host copies the chunks it wants back (the step's requests) into
//      fixed staging slots with cudaMemcpy2DAsync on a copy stream, one step
//      ahead, so the copies overlap the previous step's attention;
//   2. tiered_plan (one CTA) makes every placement decision on the device:
//      - each sequence grows by n_new tokens; a sequence entering a new chunk
//        gets a slot, and the chunk it just completed is scheduled for
//        write-back (slot -> its outbound staging slot);
//      - each request that is not resident is admitted into a slot;
//      - slots are taken free ones first (by id), then least-recently-used
//        evictable ones by (last_use, slot id); chunk 0 (the attention sink),
//        every chunk overlapping the recent window and the active chunk are
//        pinned and never evicted;
//      - the per-sequence attention tables (resident slots in chunk order)
//        and their token counts are rebuilt;
//      it emits a plan of slot-to-slot copies;
//   3. tiered_move executes the plan for all layers, K and V.
// The policy (restated in oracle/tiered_pool.py) is deterministic, so the
// resulting tables are bit-exact against the oracle.
#include "common.cuh"

namespace snapmind {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kMaxSlots = 8192;
constexpr int kMaxRequests = 64;
constexpr int kStageBatch = 4096;  // sequences whose lengths are staged in shared memory
constexpr int kAdmLog = 2048;      // slots admitted by one launch, remembered for lookups

struct PlanParams {
  int32_t* slot_owner;  // [n_slots] seq * 65536 + chunk, -1 = free
  int32_t* slot_last;   // [n_slots] step of last admission / touch
  int32_t* chunk_slot;  // [B][max_chunks] slot of a resident chunk, -1 = cold
  int32_t* seq_lens;    // [B] tokens stored
  int32_t* tables;      // [B][max_chunks] resident slots in chunk order
  int32_t* table_lens;  // [B] tokens reachable through tables
  int32_t* plan;        // [max_plan][2] (src slot, dst slot)
  int32_t* plan_count;  // [1]
  int32_t batch, max_chunks, n_slots, chunk, sink, window, step, n_new;
  int32_t stage_in_base, stage_out_base, max_plan;
  int32_t n_req;
  int32_t req_seq[kMaxRequests], req_chunk[kMaxRequests];
  int32_t* err;
};

__host__ __device__ inline int plan_sort_n(int n_slots) {
  int n = 1;
  while (n < n_slots) n <<= 1;
  return n;
}

// Shared memory of one plan launch: candidate keys [sort_n] (8 B), slot owner and
// last use [n_slots] each, then (for batches up to kStageBatch) lengths and the
// prefetched slot of each sequence's just-completed chunk [batch] each, the
// prefetched slot of each request's chunk [kMaxRequests] and the admission log.
__host__ __device__ inline size_t plan_smem_bytes(int n_slots, int batch) {
  const size_t staged = batch <= kStageBatch ? 2 * (size_t)batch : 0;
  return 8 * (size_t)plan_sort_n(n_slots) + 4 * (2 * (size_t)n_slots + staged + kMaxRequests + kAdmLog);
}

__device__ __forceinline__ bool chunk_pinned(int c, int len, int chunk, int sink, int window) {
  if (sink > 0 && c == 0) return true;                      // attention sink
  if ((int64_t)(c + 1) * chunk > (int64_t)len - window) return true;  // overlaps the recent window
  return (int64_t)(c + 1) * chunk >= len;                   // active (last, possibly partial) chunk
}

// The decisions are taken by one thread in a fixed order (the policy is sequential),
// so every value that thread reads is staged in shared memory first by the whole
// block: slot owners and last uses, sequence lengths, and the slots of the chunks
// it will look up.  A prefetched chunk -> slot entry may have changed during the
// launch; it is trusted only while the slot's owner still names the chunk, else the
// slots admitted by this launch are searched (an admitted slot is never evicted in
// the same step).  Global chunk_slot is written by that thread as it decides, so
// when the log overflows it reads its own writes back.
__global__ void __launch_bounds__(kPlanThreads) tiered_plan_kernel(PlanParams p) {
  extern __shared__ unsigned long long plan_smem[];
  const int sort_n = plan_sort_n(p.n_slots);
  const bool staged = p.batch <= kStageBatch;
  unsigned long long* cand = plan_smem;  // candidate keys, sorted ascending
  int32_t* s_owner = reinterpret_cast<int32_t*>(cand + sort_n);
  int32_t* s_last = s_owner + p.n_slots;
  int32_t* s_len = s_last + p.n_slots;                     // [batch] when staged
  int32_t* s_done = s_len + (staged ? p.batch : 0);        // [batch] when staged
  int32_t* s_req = s_done + (staged ? p.batch : 0);        // [kMaxRequests]
  int32_t* s_adm = s_req + kMaxRequests;                   // [kAdmLog]
  __shared__ int s_ncand, s_bad;
  const int tid = threadIdx.x;
  const int64_t mc = p.max_chunks;

  // ---- stage the state (coalesced, all threads)
  for (int i = tid; i < p.n_slots; i += kPlanThreads) {
    s_owner[i] = p.slot_owner[i];
    s_last[i] = p.slot_last[i];
  }
  if (staged) {
    for (int b = tid; b < p.batch; b += kPlanThreads) {
      const int old = p.seq_lens[b];
      s_len[b] = old;
      int g = -1;
      if (old > 0 && old % p.chunk == 0 && p.n_new > 0) {
        const int done = old / p.chunk - 1;
        if (done < p.max_chunks) g = p.chunk_slot[b * mc + done];
      }
      s_done[b] = g;
    }
  }
  if (tid < p.n_req) {
    const int b = p.req_seq[tid], c = p.req_chunk[tid];
    s_req[tid] = (b >= 0 && b < p.batch && c >= 0 && c < p.max_chunks) ? p.chunk_slot[b * mc + c] : -1;
  }
  if (tid == 0) {
    s_bad = 0;
  }
  __syncthreads();
  const int32_t* lens0 = staged ? s_len : p.seq_lens;

  // ---- candidate key: free slots (0, id), evictable (1 + last_use, id), others +inf.
  // Pinning is judged with the lengths after this step's growth.
  for (int s = tid; s < sort_n; s += kPlanThreads) {
    unsigned long long key = ~0ull;
    if (s < p.n_slots) {
      const int owner = s_owner[s];
      if (owner < 0) {
        key = (unsigned long long)s;
      } else {
        const int seq = owner >> 16, c = owner & 0xFFFF;
        const int len = lens0[seq] + p.n_new;
        if (!chunk_pinned(c, len, p.chunk, p.sink, p.window))
          key = ((unsigned long long)(1u + (uint32_t)s_last[s]) << 32) | (uint32_t)s;
      }
    }
    cand[s] = key;
  }
  __syncthreads();
  for (int size = 2; size <= sort_n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < sort_n; i += kPlanThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = cand[i], b = cand[j];
          if (up ? (a > b) : (a < b)) {
            cand[i] = b;
            cand[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // candidates = keys below +inf: the first index holding +inf (the keys are sorted)
  for (int i = tid; i < sort_n; i += kPlanThreads) {
    const bool here = cand[i] == ~0ull && (i == 0 || cand[i - 1] != ~0ull);
    if (here) s_ncand = i;
    if (i == sort_n - 1 && cand[i] != ~0ull) s_ncand = sort_n;
  }
  __syncthreads();

  // ---- sequential decisions (one thread, shared memory): deterministic order
  if (tid == 0) {
    int next = 0, nadm = 0, nplan = 0, bad = 0;
    bool adm_overflow = false;
    const int ncand = min(s_ncand, p.n_slots);
    // slot holding chunk c of sequence seq, or -1; g0 = its entry before this launch
    auto resident_slot = [&](int seq, int c, int g0) -> int {
      const int key = (seq << 16) | c;
      if (g0 >= 0 && g0 < p.n_slots && s_owner[g0] == key) return g0;
      if (adm_overflow) return p.chunk_slot[seq * mc + c];
      for (int a = 0; a < nadm; ++a)
        if (s_owner[s_adm[a]] == key) return s_adm[a];
      return -1;
    };
    auto take_slot = [&](int seq, int c) -> int {
      while (next < ncand) {
        const int s = (int)(cand[next++] & 0xFFFFFFFFull);
        const int owner = s_owner[s];
        if (owner >= 0) {
          if (s_last[s] == p.step) continue;  // touched or admitted in this step
          p.chunk_slot[(int64_t)(owner >> 16) * mc + (owner & 0xFFFF)] = -1;
        }
        s_owner[s] = (seq << 16) | c;
        s_last[s] = p.step;
        p.chunk_slot[seq * mc + c] = s;
        if (nadm < kAdmLog) s_adm[nadm++] = s;
        else adm_overflow = true;
        return s;
      }
      return -1;
    };
    // 1. growth: a sequence entering a new chunk needs a slot; the chunk it
    //    completed goes to its outbound staging slot
    for (int b = 0; b < p.batch; ++b) {
      const int old = staged ? s_len[b] : p.seq_lens[b];
      const int len = old + p.n_new;
      const int c_first = (old + p.chunk - 1) / p.chunk;   // first chunk not yet allocated
      const int c_last = (len + p.chunk - 1) / p.chunk;    // chunks needed after growth
      if (old > 0 && old % p.chunk == 0 && p.n_new > 0) {
        const int done = old / p.chunk - 1;
        if (done < p.max_chunks) {
          const int src = resident_slot(b, done, staged ? s_done[b] : p.chunk_slot[b * mc + done]);
          if (src >= 0 && nplan < p.max_plan) {
            p.plan[2 * nplan] = src;
            p.plan[2 * nplan + 1] = p.stage_out_base + b;
            ++nplan;
          }
        }
      }
      for (int c = c_first; c < c_last; ++c) {
        if (c >= p.max_chunks || c > 0xFFFF) {
          bad |= SNAPMIND_DEVERR_TABLE;
          break;
        }
        if (take_slot(b, c) < 0) bad |= SNAPMIND_DEVERR_OUT_OF_BLOCKS;
      }
      p.seq_lens[b] = len;
      if (staged) s_len[b] = len;
    }
    // 2. requests
    for (int i = 0; i < p.n_req; ++i) {
      const int b = p.req_seq[i], c = p.req_chunk[i];
      if (b < 0 || b >= p.batch) continue;
      const int len = staged ? s_len[b] : p.seq_lens[b];
      if (c < 0 || c >= p.max_chunks || (int64_t)c * p.chunk >= len) continue;
      const int cur = resident_slot(b, c, s_req[i]);
      if (cur >= 0) {
        s_last[cur] = p.step;  // already resident: touch
        continue;
      }
      const int s = take_slot(b, c);
      if (s < 0) {
        bad |= SNAPMIND_DEVERR_OUT_OF_BLOCKS;
        continue;
      }
      if (nplan < p.max_plan) {
        p.plan[2 * nplan] = p.stage_in_base + i;
        p.plan[2 * nplan + 1] = s;
        ++nplan;
      }
    }
    *p.plan_count = nplan;
    s_bad = bad;
  }
  __syncthreads();

  // ---- write the slot state back
  for (int i = tid; i < p.n_slots; i += kPlanThreads) {
    p.slot_owner[i] = s_owner[i];
    p.slot_last[i] = s_last[i];
  }

  // ---- 3. attention tables: one warp per sequence, ballot compaction in chunk order;
  // each lane loads its 4 entries of a 128-chunk group before using any of them
  const int warp = tid >> 5, lane = tid & 31;
  for (int b = warp; b < p.batch; b += kPlanThreads / 32) {
    const int len = staged ? s_len[b] : p.seq_lens[b];
    const int nchunks = min(p.max_chunks, (len + p.chunk - 1) / p.chunk);
    const int32_t* row = p.chunk_slot + b * mc;
    int n = 0, tokens = 0;
    for (int c0 = 0; c0 < nchunks; c0 += 128) {
      int sv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = c0 + 32 * k + lane;
        sv[k] = c < nchunks ? row[c] : -1;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = c0 + 32 * k + lane;
        const unsigned mask = __ballot_sync(0xffffffffu, sv[k] >= 0);
        if (sv[k] >= 0) {
          p.tables[b * mc + n + __popc(mask & ((1u << lane) - 1))] = sv[k];
          tokens += min(p.chunk, len - c * p.chunk);
        }
        n += __popc(mask);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) tokens += __shfl_xor_sync(0xffffffffu, tokens, off);
    if (lane == 0) p.table_lens[b] = tokens;
  }
  if (tid == 0 && s_bad) flag_error(p.err, s_bad);
}

struct MoveParams {
  char* pool[2];
  int64_t layer_stride;  // bytes
  int64_t slot_bytes;    // bytes of one slot in one layer (H x chunk x D)
  int32_t n_layers;
  const int32_t* plan;
  const int32_t* plan_count;
  int32_t max_plan;
};

// grid: (max_plan, n_layers, 2); each CTA copies one (entry, layer, K|V) slot
__global__ void __launch_bounds__(256) tiered_move_kernel(MoveParams p) {
  const int e = blockIdx.x, layer = blockIdx.y, kv = blockIdx.z;
  if (e >= *p.plan_count) return;
  const int src = p.plan[2 * e], dst = p.plan[2 * e + 1];
  const char* base = (kv ? p.pool[1] : p.pool[0]) + layer * p.layer_stride;  // no local copy of the array
  const Vec16* s = reinterpret_cast<const Vec16*>(base + src * p.slot_bytes);
  Vec16* d = reinterpret_cast<Vec16*>(const_cast<char*>(base) + dst * p.slot_bytes);
  const int n = (int)(p.slot_bytes / 16);
  for (int i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
}

}  // namespace
}  // namespace snapmind

using namespace snapmind;

extern "C" {

int snapmind_tiered_plan(int32_t* slot_owner, int32_t* slot_last, int32_t* chunk_slot, int32_t* seq_lens,
                         int32_t* tables, int32_t* table_lens, int32_t* plan, int32_t* plan_count, int32_t batch,
                         int32_t max_chunks, int32_t n_slots, int32_t chunk, int32_t sink, int32_t window,
                         int32_t step, int32_t n_new, int32_t stage_in_base, int32_t stage_out_base,
                         int32_t max_plan, const int32_t* req_seq, const int32_t* req_chunk, int32_t n_req,
                         int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(batch > 0 && batch <= 65535 && max_chunks > 0 && max_chunks <= 65536 && n_slots > 0 &&
                         n_slots <= kMaxSlots && chunk > 0 && sink >= 0 && window >= 0 && n_new >= 0 &&
                         max_plan > 0 && step >= 0,
                     "tiered_plan: bad sizes (n_slots <= %d)", kMaxSlots);
  SNAPMIND_CHECK_ARG(n_req >= 0 && n_req <= kMaxRequests, "tiered_plan: at most %d requests", kMaxRequests);
  SNAPMIND_CHECK_ARG(slot_owner && slot_last && chunk_slot && seq_lens && tables && table_lens && plan && plan_count,
                     "tiered_plan: null pointer");
  PlanParams p;
  p.slot_owner = slot_owner;
  p.slot_last = slot_last;
  p.chunk_slot = chunk_slot;
  p.seq_lens = seq_lens;
  p.tables = tables;
  p.table_lens = table_lens;
  p.plan = plan;
  p.plan_count = plan_count;
  p.batch = batch;
  p.max_chunks = max_chunks;
  p.n_slots = n_slots;
  p.chunk = chunk;
  p.sink = sink;
  p.window = window;
  p.step = step;
  p.n_new = n_new;
  p.stage_in_base = stage_in_base;
  p.stage_out_base = stage_out_base;
  p.max_plan = max_plan;
  p.n_req = n_req;
  for (int i = 0; i < n_req; ++i) {
    p.req_seq[i] = req_seq[i];
    p.req_chunk[i] = req_chunk[i];
  }
  p.err = err_word;
  const size_t smem = plan_smem_bytes(n_slots, batch);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(tiered_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "tiered_plan smem attribute");
  }
  tiered_plan_kernel<<<1, kPlanThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
  SNAPMIND_LAUNCH_CHECK("tiered_plan launch");
}

int snapmind_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width,
                     int64_t height, void* stream) {
  SNAPMIND_CHECK_ARG(dst && src && width >= 0 && height >= 0 && dst_pitch >= width && src_pitch >= width,
                     "copy_2d: bad arguments");
  if (width == 0 || height == 0) return SNAPMIND_OK;
  return cuda_status(cudaMemcpy2DAsync(dst, (size_t)dst_pitch, src, (size_t)src_pitch, (size_t)width, (size_t)height,
                                       cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
                     "copy_2d");
}

int snapmind_tiered_move(void* k_pool, void* v_pool, int64_t layer_stride_bytes, int64_t slot_bytes,
                         int32_t n_layers, const int32_t* plan, const int32_t* plan_count, int32_t max_plan,
                         void* stream) {
  SNAPMIND_CHECK_ARG(n_layers > 0 && n_layers <= 65535 && max_plan > 0 && slot_bytes > 0 && slot_bytes % 16 == 0,
                     "tiered_move: bad sizes (slot bytes must be a multiple of 16)");
  SNAPMIND_CHECK_ARG(k_pool && v_pool && plan && plan_count, "tiered_move: null pointer");
  SNAPMIND_CHECK_ARG((reinterpret_cast<uintptr_t>(k_pool) & 15) == 0 && (reinterpret_cast<uintptr_t>(v_pool) & 15) == 0 &&
                         layer_stride_bytes % 16 == 0,
                     "tiered_move: pools must be 16-byte aligned");
  MoveParams p{{static_cast<char*>(k_pool), static_cast<char*>(v_pool)}, layer_stride_bytes, slot_bytes, n_layers,
               plan, plan_count, max_plan};
  dim3 grid(max_plan, n_layers, 2);
  tiered_move_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  SNAPMIND_LAUNCH_CHECK("tiered_move launch");
}

}  // extern "C"
