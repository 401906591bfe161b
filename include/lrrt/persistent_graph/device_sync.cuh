// sm_100a synchronisation and bulk-copy primitives used by the resident
// schedulers and workloads: gpu-scope acquire/release accesses, %globaltimer
// deadlines, mbarriers and TMA copies into this CTA's own shared memory
// (every copy has exactly one destination CTA).
#ifndef LRRT_PERSISTENT_GRAPH_DEVICE_SYNC_CUH_
#define LRRT_PERSISTENT_GRAPH_DEVICE_SYNC_CUH_

#include <cstdint>

namespace lrrt::persistent_graph::device {

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t value;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(value));
  return value;
}

__device__ __forceinline__ uint32_t dynamic_shared_bytes() {
  uint32_t value;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(value));
  return value;
}

__device__ __forceinline__ uint32_t load_acquire(const uint32_t *address) {
  uint32_t value;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];"
               : "=r"(value)
               : "l"(address)
               : "memory");
  return value;
}

__device__ __forceinline__ uint32_t load_relaxed(const uint32_t *address) {
  uint32_t value;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];"
               : "=r"(value)
               : "l"(address)
               : "memory");
  return value;
}

__device__ __forceinline__ void store_release(uint32_t *address, uint32_t value) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(address), "r"(value)
               : "memory");
}

__device__ __forceinline__ uint32_t fetch_add_acq_rel(uint32_t *address,
                                                      uint32_t value) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(address), "r"(value)
               : "memory");
  return old;
}

__device__ __forceinline__ void add_release(uint32_t *address, uint32_t value) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(address), "r"(value)
               : "memory");
}

// Wait limit helper: every spin in the resident kernels compares against a
// deadline taken from the launch's wait limit. The clock starts at the first
// check: a wait that never has to check (the common case) reads no timer, and
// constructing one stalls no warp on a special-register read.
struct Deadline {
  mutable uint64_t end_ns;
  uint32_t limit_ms;
  __device__ __forceinline__ explicit Deadline(uint32_t limit) : end_ns(0), limit_ms(limit) {}
  __device__ __forceinline__ bool expired() const {
    const uint64_t now = global_timer_ns();
    if (end_ns == 0) {
      end_ns = now + uint64_t{limit_ms} * 1000000ull;
      return false;
    }
    return now > end_ns;
  }
};

// ---- mbarrier + TMA bulk copy --------------------------------------------

__device__ __forceinline__ uint32_t shared_address(const void *pointer) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(pointer));
}

__device__ __forceinline__ void mbarrier_init(uint64_t *barrier, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(
                   shared_address(barrier)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbarrier_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbarrier_arrive_expect_tx(uint64_t *barrier,
                                                          uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
          shared_address(barrier)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbarrier_try_wait(uint64_t *barrier,
                                                  uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(shared_address(barrier)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on an mbarrier phase; false when the deadline passed first.
__device__ __forceinline__ bool mbarrier_wait(uint64_t *barrier, uint32_t parity,
                                              const Deadline &deadline) {
  uint32_t spins = 0;
  while (!mbarrier_try_wait(barrier, parity)) {
    if ((++spins & 255u) == 0u && deadline.expired()) {
      return false;
    }
  }
  return true;
}

// Global -> shared bulk copy completing on `barrier`. Addresses 16-byte
// aligned, bytes a multiple of 16. Uses an evict-first L2 policy: weights are
// streamed once per decode step and should not displace reused data.
__device__ __forceinline__ void bulk_copy_to_shared(void *destination,
                                                    const void *source,
                                                    uint32_t bytes,
                                                    uint64_t *barrier,
                                                    uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(shared_address(destination)),
      "l"(source), "r"(bytes), "r"(shared_address(barrier)), "l"(policy)
      : "memory");
}

// 2-D TMA tile load of the box at (x, y) of the tensor map `map` (a
// CUtensorMap in global memory) into shared memory, completing on `barrier`.
// One destination CTA. x times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tensor_load_2d(void *destination, const void *map, uint32_t x,
                                               uint32_t y, uint64_t *barrier) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(shared_address(destination)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(shared_address(barrier))
      : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(policy));
  return policy;
}

// ---- exchange words ---------------------------------------------------------
// A value published to other blocks together with its readiness: one 64-bit
// word tag << 32 | float bits, written and read as single 64-bit accesses
// (single-copy atomic), so a reader that sees the tag it waits for also sees
// the value stored with it, without fences or a separate flag.

__device__ __forceinline__ uint64_t exchange_word(float value, uint32_t tag) {
  return (uint64_t{tag} << 32) | __float_as_uint(value);
}

__device__ __forceinline__ void exchange_store(uint64_t *word, float value, uint32_t tag) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(word),
               "l"(exchange_word(value, tag))
               : "memory");
}

// Two consecutive words (16-byte aligned) in one access; each word is
// single-copy atomic on its own.
__device__ __forceinline__ void exchange_store2(uint64_t *word, float first, float second,
                                                uint32_t tag) {
  asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(word),
               "l"(exchange_word(first, tag)), "l"(exchange_word(second, tag))
               : "memory");
}

// Two consecutive words (16-byte aligned).
__device__ __forceinline__ void exchange_load2(const uint64_t *word, uint64_t &first,
                                               uint64_t &second) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];"
               : "=l"(first), "=l"(second)
               : "l"(word));
}

__device__ __forceinline__ uint32_t exchange_tag(uint64_t word) {
  return static_cast<uint32_t>(word >> 32);
}

__device__ __forceinline__ float exchange_value(uint64_t word) {
  return __uint_as_float(static_cast<uint32_t>(word));
}

// L2-coherent loads for data other blocks wrote during this kernel.
__device__ __forceinline__ float load_cg(const float *address) {
  return __ldcg(address);
}
__device__ __forceinline__ float4 load_cg4(const float *address) {
  return __ldcg(reinterpret_cast<const float4 *>(address));
}
__device__ __forceinline__ uint32_t load_cg(const uint32_t *address) {
  return __ldcg(address);
}

} // namespace lrrt::persistent_graph::device

#endif // LRRT_PERSISTENT_GRAPH_DEVICE_SYNC_CUH_
