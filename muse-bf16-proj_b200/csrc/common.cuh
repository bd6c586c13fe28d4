// Shared device helpers for the B200 (sm_100a) small-M projection library.
//
// Everything here is hand-written inline PTX or plain CUDA C++: mbarriers, 1-D bulk copies (TMA engine, no
// tensor map), thread-block-cluster distributed shared memory, mma.sync, and the 12-bit weight decode.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/mbp.h"

#define MBP_DEV __device__ __forceinline__

namespace mbp {

// ------------------------------------------------------------------------------------------------------------
// device status word: bounded waits record why they gave up instead of trapping
// ------------------------------------------------------------------------------------------------------------
// One status word per translation unit (no relocatable device code); mbp_status ORs them together through
// each unit's read_status_here().
static __device__ int g_status = 0;

static inline int read_status_here(int* v, int clear) {
  int x = 0;
  if (cudaMemcpyFromSymbol(&x, g_status, sizeof(int)) != cudaSuccess) return MBP_ERR_LAUNCH;
  if (x && !*v) *v = x;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_status, &z, sizeof(int)) != cudaSuccess) return MBP_ERR_LAUNCH;
  }
  return MBP_OK;
}

MBP_DEV void set_status(int code) { atomicCAS(&g_status, 0, code); }

MBP_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Limit of every bounded wait.  Each launch copies the library-wide setting (mbp_set_wait_limit, default 1 s: a
// wait this long means a lost arrival) into its parameters, so a kernel captured in a CUDA graph keeps the limit
// in force when it was captured.
constexpr uint64_t kDefaultWaitLimitNs = 1000000000ull;
uint64_t wait_limit_ns();  // host: the current setting (abi.cu)

// Single-copy-atomic 64-bit accesses at system scope (epoch-tagged words exchanged between GPUs).
MBP_DEV void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
MBP_DEV uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait for an exchange word tagged with epoch e (tag in the upper 32 bits; data and tag arrive in one
// store).  t0 = 0 on the first call of a thread; once `limit` ns have passed since then the status word gets
// MBP_DEV_TIMEOUT_PEER and `dead` stops further waits of the thread (the words are then read as they are).
MBP_DEV uint64_t wait_tag(const uint64_t* p, uint32_t e, uint64_t& t0, bool& dead, uint64_t limit) {
  uint64_t v = ld_relaxed_sys_u64(p);
  while ((uint32_t)(v >> 32) != e && !dead) {
    const uint64_t now = globaltimer();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > limit) {
      set_status(MBP_DEV_TIMEOUT_PEER);
      dead = true;
    }
    __nanosleep(32);
    v = ld_relaxed_sys_u64(p);
  }
  return v;
}

// ------------------------------------------------------------------------------------------------------------
// shared memory / mbarrier
// ------------------------------------------------------------------------------------------------------------
MBP_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MBP_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

MBP_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

MBP_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive that cannot issue before `dep` is available.  A consumer handing a TMA-filled stage back passes a value
// computed from everything it read from the stage: its shared loads have then completed, so the producer's next
// copy into the stage cannot overwrite data a load has not yet returned (the arrive itself does not wait for
// outstanding loads).
MBP_DEV void mbar_arrive_dep(uint32_t bar, uint32_t dep) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar), "r"(dep) : "memory");
}

MBP_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

MBP_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase completes or `ns` elapse,
// instead of spinning through the issue slots of the warps that do the work.
MBP_DEV bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code`) if the phase did not complete within `limit` ns.
MBP_DEV bool mbar_wait(uint32_t bar, uint32_t parity, int code, uint64_t limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
    if (globaltimer() - t0 > limit) {
      set_status(code);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared through the TMA engine, completing bytes on an mbarrier.
// dst, src 16-byte aligned; bytes a multiple of 16.
MBP_DEV void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Same with an L2 cache policy (evict-first for streamed weights).
MBP_DEV void bulk_g2s_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// 2-D tiled TMA load of box {x, y} into this CTA's shared memory, from a tensor map in kernel-parameter space.
MBP_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

MBP_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Bulk prefetch of global memory into L2 (a hint: no completion, no ordering).  src 16-byte aligned, bytes % 16 == 0.
MBP_DEV void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch.  grid_dep_wait returns once every grid this one depends on has completed and
// its memory is visible (immediately when the launch had no programmatic dependency); grid_dep_launch lets the
// next grid of the stream be scheduled once every CTA of this grid has called it or exited.
MBP_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MBP_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

MBP_DEV uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

MBP_DEV uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

MBP_DEV uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

MBP_DEV void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Named barrier over `count` threads (multiple of 32), id 1..15 (0 is __syncthreads).
MBP_DEV void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------------------------------------------------------------------
// thread-block cluster
// ------------------------------------------------------------------------------------------------------------
MBP_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Non-.aligned forms: correct even if a warp reaches the barrier diverged (every thread still arrives once).
MBP_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
MBP_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
MBP_DEV void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}

MBP_DEV uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}

MBP_DEV void st_dsmem_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

MBP_DEV float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

// ------------------------------------------------------------------------------------------------------------
// tensor core (legacy warp-level path): D += A(16x16 bf16) * B(16x8 bf16), FP32 accumulate
// ------------------------------------------------------------------------------------------------------------
// Not volatile: a pure function of its operands, so the scheduler may interleave it with loads of later units.
MBP_DEV void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                            uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------------------------------------------------
// 12-bit decode.  A unit is 16 rows x 64 columns; lane l = 4g + t holds 32 values v = 8q + 4hf + 2rh + d at
// row 8rh + g, column 16t + 4q + 2hf + d.  Plane 0 (bytes 0-511) and plane 1 (512-1023) hold the low bytes
// of values 0-15 / 16-31, lane-major (16 bytes per lane); plane 2 (1024-1535) holds 4 code words per lane.
// Code word w covers values 8w..8w+7: a 3-bit exponent offset at nibble i, the sign of value i at bit
// kSignPos[i] = {3,19,7,23,11,27,15,31}[i].  Decoded register A[4q + 2hf + rh] is the bf16x2 pair (d = 0, 1),
// i.e. the mma.sync m16n8k16 A fragment of k-step q.
// ------------------------------------------------------------------------------------------------------------
MBP_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Decodes the 8 weights of one k-step.  L0 / L1 carry the low bytes of weights 0-3 / 4-7 and C their code
// word.  The 3-bit exponent offsets of C, masked to nibbles, select through prmt a byte of the 8-entry table T0:T1
// (exponent bytes base .. base+7); a second prmt interleaves those high bytes with the low bytes into bf16 pairs
// in the A-fragment order, and the sign bits are moved from their code-word positions to bit 15 of each half.
MBP_DEV void decode8(uint32_t L0, uint32_t L1, uint32_t C, uint32_t T0, uint32_t T1, uint32_t* a) {
  const uint32_t cm = C & 0x77777777u;
  const uint32_t h0 = prmt(T0, T1, cm);
  const uint32_t h1 = prmt(T0, T1, cm >> 16);
  a[0] = prmt(L0, h0, 0x5140u) | ((C << 12) & 0x80008000u);
  a[1] = prmt(L0, h0, 0x7362u) | ((C << 8) & 0x80008000u);
  a[2] = prmt(L1, h1, 0x5140u) | ((C << 4) & 0x80008000u);
  a[3] = prmt(L1, h1, 0x7362u) | (C & 0x80008000u);
}

MBP_DEV void decode_unit(const uint4& p0, const uint4& p1, const uint4& p2, uint32_t T0, uint32_t T1,
                         uint32_t (&A)[16]) {
  decode8(p0.x, p0.y, p2.x, T0, T1, A + 0);
  decode8(p0.z, p0.w, p2.y, T0, T1, A + 4);
  decode8(p1.x, p1.y, p2.z, T0, T1, A + 8);
  decode8(p1.z, p1.w, p2.w, T0, T1, A + 12);
}

// decode8 with escape restoration: X0/X1 hold the exponent XOR bytes of values 0-3 / 4-7 (the byte order of the
// table lookups h0/h1), applied to the high bytes before the sign is merged.
MBP_DEV void decode8m(uint32_t L0, uint32_t L1, uint32_t C, uint32_t T0, uint32_t T1, uint32_t X0, uint32_t X1,
                      uint32_t* a) {
  const uint32_t cm = C & 0x77777777u;
  const uint32_t h0 = prmt(T0, T1, cm) ^ X0;
  const uint32_t h1 = prmt(T0, T1, cm >> 16) ^ X1;
  a[0] = prmt(L0, h0, 0x5140u) | ((C << 12) & 0x80008000u);
  a[1] = prmt(L0, h0, 0x7362u) | ((C << 8) & 0x80008000u);
  a[2] = prmt(L1, h1, 0x5140u) | ((C << 4) & 0x80008000u);
  a[3] = prmt(L1, h1, 0x7362u) | (C & 0x80008000u);
}

// decode_unit with the lane's two unit-mask words (m0 = values 0-15, m1 = values 16-31, one byte per value).
MBP_DEV void decode_unit_m(const uint4& p0, const uint4& p1, const uint4& p2, uint32_t T0, uint32_t T1,
                           const uint4& m0, const uint4& m1, uint32_t (&A)[16]) {
  decode8m(p0.x, p0.y, p2.x, T0, T1, m0.x, m0.y, A + 0);
  decode8m(p0.z, p0.w, p2.y, T0, T1, m0.z, m0.w, A + 4);
  decode8m(p1.x, p1.y, p2.z, T0, T1, m1.x, m1.y, A + 8);
  decode8m(p1.z, p1.w, p2.w, T0, T1, m1.z, m1.w, A + 12);
}

MBP_DEV uint32_t table_lo(uint32_t base) { return base * 0x01010101u + 0x03020100u; }
MBP_DEV uint32_t table_hi(uint32_t base) { return base * 0x01010101u + 0x07060504u; }

// Escape entry: chunk << 17 | lane << 12 | value << 7 | xor7 (XOR of the 7 high exponent bits).
MBP_DEV uint32_t esc_chunk(uint32_t e) { return e >> 17; }
MBP_DEV uint32_t esc_lane(uint32_t e) { return (e >> 12) & 31u; }
MBP_DEV uint32_t esc_value(uint32_t e) { return (e >> 7) & 31u; }

}  // namespace mbp
