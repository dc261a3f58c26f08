// Tensor parallelism over NVLink peer memory (one process per GPU, Megatron split).
//
// Each rank allocates one region of device memory and exports it with a CUDA IPC handle;
// every rank maps every peer's region. The region holds:
//   flags[slot][src]  u64, the epoch at which rank `src` last signalled `slot`
//                     (written by the peer with a system-scope release store);
//   bulk parts        [2 parities][MAX_M * hidden] f32: the prefill allreduce's input;
//   ll                [2 parities][src][4 tokens][rows] u64: row-parallel GEMV partials
//                     pushed by each peer, each value tagged with its exchange's epoch;
//   llkeys            [3 sets][2 rows][src][2] u64: the greedy argmax candidates, tagged
//                     alike (set 0: forward steps; sets 1, 2: MTP drafts, alternately);
//   logits            [2 rows][vocab / N] f32: this rank's LM-head shard.
// The decode exchanges (GEMV partials, argmax keys) use tagged words: the writer stores
// (epoch << 32 | value) into the peer's memory with one 64-bit system-scope store, and
// the reader polls its own memory until the tag matches, so no fence and no remote load
// is on the path. The bulk exchanges (prefill partials, gathered logits) publish data and
// then a flag.
// An exchange at site s of step t uses epoch t * sites + s + 1, so flags only grow and
// never need resetting. Data buffers alternate by epoch parity: a rank rewrites a buffer
// two exchanges later, and by then every peer has signalled the exchange in between,
// which it does only after it has finished reading. Every wait is bounded by the global
// timer (TpComm::wait_ns, 2 s unless SNL_TP_WAIT_MS says otherwise); one that runs out
// sets bit 1 of the device error word and the kernel carries on. A wait that finds bit 1
// already set gives up at once, so a dead peer costs one bound per step, not one per wait.
// An MTP draft (replicated MTP layer, vocabulary-split head) is a step of its own: its
// embedding advances the counter, and its only exchange is the argmax. Two drafts may
// follow each other with no other exchange between them, so drafts alternate between two
// key slot sets of their own: a set is rewritten only after the other set's exchange,
// which every peer joins after reading the first.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace snl {

constexpr int kTpMax = 8;
constexpr uint32_t kTpSlots = 1024;  // flag slots per rank
constexpr unsigned long long kTpWaitNs = 2000000000ull;  // default bound of one cross-GPU wait
// Argmax key slots: [kTpKeySets][kTpKeyRows][src][2] tagged words per rank.
constexpr uint32_t kTpKeySets = 3;
constexpr uint32_t kTpKeyRows = 2;

// Device view of the communicator (passed by value to kernels).
struct TpComm {
  int rank = 0, size = 1;
  uint64_t* flags[kTpMax] = {};     // each rank's flag array, [kTpSlots][kTpMax]
  float* bparts[kTpMax] = {};       // each rank's bulk partials, [2][bp_elems]
  unsigned long long* ll[kTpMax] = {};      // each rank's tagged GEMV partials, [2][kTpMax][4][gp_rows]
  unsigned long long* llkeys[kTpMax] = {};  // each rank's tagged argmax keys, [2 rows][kTpMax][2]
  float* logits[kTpMax] = {};       // each rank's LM-head shard, [2][vocab_local]
  uint32_t gp_rows = 0;
  uint64_t bp_elems = 0;
  const unsigned long long* step = nullptr;  // device step counter (this rank)
  uint32_t sites = 1;                        // exchanges per step
  int* err = nullptr;
  unsigned long long wait_ns = kTpWaitNs;    // bound of every wait, in global-timer ns
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// True once some wait of this device has given up (bit 1 of the error word).
__device__ __forceinline__ bool tp_gave_up(const TpComm& c) { return (*(volatile const int*)c.err & 2) != 0; }

__device__ __forceinline__ uint64_t tp_epoch(const TpComm& c, uint32_t site) {
  return *(volatile const unsigned long long*)c.step * c.sites + site + 1;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ld_cv(const float* p) {
  float v;
  asm volatile("ld.global.cv.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_cv_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.cv.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Signal `slot` at `epoch` to every rank (including this one). Call after this thread's
// data stores, from one thread; preceded by a system-scope fence.
__device__ __forceinline__ void tp_signal(const TpComm& c, uint32_t slot, uint64_t epoch) {
  __threadfence_system();
  for (int q = 0; q < c.size; q++) st_release_sys(c.flags[q] + (uint64_t)slot * kTpMax + c.rank, epoch);
}

// Wait until rank `src` has signalled `slot` at `epoch` or later. False if the bound ran out.
__device__ __forceinline__ bool tp_wait_one(const TpComm& c, uint32_t slot, int src, uint64_t epoch) {
  const uint64_t* f = c.flags[c.rank] + (uint64_t)slot * kTpMax + src;
  if (ld_acquire_sys(f) >= epoch) return true;
  if (tp_gave_up(c)) return false;
  const unsigned long long t0 = global_ns();
  while (ld_acquire_sys(f) < epoch) {
    if (tp_gave_up(c)) return false;
    if (global_ns() - t0 > c.wait_ns) {
      atomicOr(c.err, 2);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ll_word(uint32_t tag, uint32_t bits) {
  return ((unsigned long long)tag << 32) | bits;
}
// Polls a tagged word of this rank's memory until its tag is `tag`; returns the value
// bits, or sets bit 1 of the error word and returns 0 when the bound runs out (at once
// when another wait already gave up).
__device__ __forceinline__ uint32_t ll_wait(const TpComm& c, const unsigned long long* p, uint32_t tag) {
  unsigned long long w = ld_relaxed_sys_u64(p);
  if ((uint32_t)(w >> 32) == tag) return (uint32_t)w;
  if (tp_gave_up(c)) return 0u;
  const unsigned long long t0 = global_ns();
  for (;;) {
    w = ld_relaxed_sys_u64(p);
    if ((uint32_t)(w >> 32) == tag) return (uint32_t)w;
    if (tp_gave_up(c)) return 0u;
    if (global_ns() - t0 > c.wait_ns) {
      atomicOr(c.err, 2);
      return 0u;
    }
  }
}

// Host side.
struct TpHost {
  int rank = 0, size = 1;
  void* region = nullptr;       // this rank's exported region
  size_t region_bytes = 0;
  void* peer_base[kTpMax] = {};  // mapped regions (own at [rank])
  bool connected = false;
  // offsets inside a region
  size_t off_flags = 0, off_bparts = 0, off_ll = 0, off_llkeys = 0, off_logits = 0;
  TpComm comm;
};

// Flag slots of the bulk exchanges.
constexpr uint32_t kSlotBulk = kTpSlots - 1;
constexpr uint32_t kSlotLogits = kTpSlots - 2;

// Exchange kernels (tp.cu).
// Sums every rank's bulk partial [n] (parity of the site's epoch) in rank order into out.
int launch_tp_allreduce(const TpComm& c, uint32_t site, uint64_t n, float* out, cudaStream_t s);
// Copies every rank's LM-head shard [rows][vl] into full[rows][vl * size].
int launch_tp_gather_logits(const TpComm& c, uint32_t site, uint32_t rows, uint32_t vl, float* full, cudaStream_t s);
// Greedy argmax over an LM-head shard [rows][vl] agreed by all ranks (layers.cu), through
// key slot set key_set (0: forward steps; 1 and 2, alternately: MTP drafts).
int launch_argmax_tp(const float* logits, uint32_t rows, uint32_t vl, uint32_t* out_idx, unsigned long long* part,
                     const TpComm& c, uint32_t site, cudaStream_t s, uint32_t key_set = 0);

}  // namespace snl
