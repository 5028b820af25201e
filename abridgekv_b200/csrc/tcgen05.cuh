// tcgen05 / TMA building blocks shared by the attention kernels on sm_100a
// (prefill.cu: dense masked prefill; codestep.cu: paged code step): UMMA shared
// memory descriptors and instruction descriptors, tcgen05.mma / commit /
// ld / st / fences, 4D tensor-map copies, bounded mbarrier waits, packed fp32
// helpers for the softmax, and the host-side tensor-map encoder.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace abkv {
namespace tc {

// Packed fp32 pairs (sm_100 f32x2 pipes) and a three-input max: fewer issue
// slots per score in the softmax.
static __device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n .reg .b64 x, y, z, r;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %4};\n mov.b64 z, {%5, %5};\n"
      " fma.rn.f32x2 r, x, y, z;\n mov.b64 {%0, %1}, r;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
static __device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1) {
  asm("{\n .reg .b64 x, y, r;\n mov.b64 x, {%0, %1};\n mov.b64 y, {%2, %3};\n"
      " add.rn.f32x2 r, x, y;\n mov.b64 {%0, %1}, r;\n}\n"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1));
}
static __device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

static __device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// ---- tcgen05 / TMA helpers --------------------------------------------------
static __device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t saddr) {
  // K-major, 128B swizzle: rows of 128 B, 8-row atoms 1024 B apart (SBO),
  // LBO unused (1), descriptor version 1, layout type 2 (SWIZZLE_128B).
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
static __device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t saddr, uint32_t lbo) {
  // MN-major, 128B swizzle: a K row = 64 MN elements (128 B); 8 K rows form a
  // 1024 B atom (SBO = 1024); the next 64 MN elements are `lbo` bytes away.
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// The descriptor of the same operand `bytes` further on in shared memory (bytes a
// multiple of 16).  Shared memory addresses stay below 256 KiB, so the 14-bit
// start-address field (address >> 4) cannot carry into the next field: one add
// instead of rebuilding the descriptor for every instruction of an unrolled loop.
static __device__ __forceinline__ uint64_t desc_advance(uint64_t desc, uint32_t bytes) { return desc + (bytes >> 4); }
// kind::f16 instruction descriptor: D f32 (bit 4), A and B bf16 (bits 7, 10),
// B MN-major if b_mn_major (bit 16; A is K-major), N >> 3 at bit 17, M >> 4 at
// bit 24 (M = 128).
constexpr uint32_t idesc_bf16_m128(uint32_t n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major ? (1u << 16) : 0u) | ((n >> 3) << 17) |
         ((128u >> 4) << 24);
}

static __device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// A operand from TMEM (128 lanes x 16 bf16 = 8 columns per K step of 16).
static __device__ __forceinline__ void umma_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
static __device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}
static __device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
static __device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
static __device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
static __device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// Named barrier of `count` threads (whole warps) other than the CTA-wide barrier 0.
static __device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}
// Named barrier that also ANDs a per-thread flag over its `count` threads: every participant gets
// the same answer, so warps that must stay in step take an early exit together.
static __device__ __forceinline__ bool named_bar_and(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred q, o;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred o, %2, %3, q;\n selp.u32 %0, 1, 0, o;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

static __device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
static __device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
static __device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

static __device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
// Shared -> global tensor store of one box (no multicast), tracked by the issuing thread's bulk
// async-group: commit it, then wait for its reads before the shared memory is reused or the CTA exits.
static __device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
static __device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
static __device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
}
// Eight bf16 (four words) into row `row` of a [rows][128 B] 128B-swizzled shared-memory atom at
// 16-byte chunk `chunk` (0..7): the layout a SWIZZLE_128B tensor map reads.
static __device__ __forceinline__ void st_swizzled16(uint8_t* atom, int row, int chunk, uint32_t a, uint32_t b,
                                              uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(smem_u32(atom + row * 128 + ((chunk ^ (row & 7)) << 4))),
               "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// Bounded wait; after the first expiry a thread stops waiting altogether (its
// remaining work is skipped and the error word says why), so a fault in one
// role cannot stall the CTA for long.
static __device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, bool& dead, int32_t* err) {
  if (dead) return false;
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < (1u << 20); ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  set_error(err, ABKV_DEVERR_TIMEOUT);
  dead = true;
  return false;
}

static __device__ __forceinline__ void mbar_arrive_one(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}



// Online-softmax state of one query row.
struct SoftmaxState {
  float m_run, l_run;
};

// ---- host -------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Tiled tensor map of rank 1..5 with byte strides gstr (dims 1..rank-1).  The
// driver entry point is resolved through the runtime, so the library does not
// link libcuda and still loads on hosts without a GPU driver.
static inline int encode_tiled(CUtensorMap* m, CUtensorMapDataType dtype, int rank, const void* base,
                               const cuuint64_t* dims, const cuuint64_t* gstr, const cuuint32_t* box,
                               CUtensorMapSwizzle swizzle) {
  if (rank < 2 || rank > 5) return ABKV_ERR_INVALID_ARG;
  // gstr[i] is the byte stride of dimension i + 1.  A dimension of extent 1 is never stepped
  // through, so its stride addresses nothing (torch and numpy give such dimensions stride 0 after
  // unsqueeze / expand, which the encoder rejects): replace it with the packed extent of the
  // dimensions inside it, a legal value.
  const size_t esize = dtype == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  cuuint64_t g[4];
  for (int i = 0; i < rank - 1; ++i) {
    g[i] = gstr[i];
    if (dims[i + 1] == 1) {
      const cuuint64_t packed = i == 0 ? dims[0] * esize : g[i - 1] * dims[i];
      g[i] = (packed + 15) / 16 * 16;
    }
    if (g[i] % 16 != 0 || g[i] == 0) return ABKV_ERR_INVALID_ARG;
  }
  gstr = g;
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  // cuTensorMapEncodeTiled is a driver call: it needs the device's context current in the calling
  // thread, which a thread that made no runtime call yet (autograd's device thread, a worker
  // pool) does not have.  cudaFree(nullptr) binds the primary context; once per thread and device.
  static thread_local int bound_device = -1;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return ABKV_ERR_CUDA;
  if (bound_device != device) {
    if (cudaFree(nullptr) != cudaSuccess) return ABKV_ERR_CUDA;
    bound_device = device;
  }
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) != cudaSuccess ||
      qres != cudaDriverEntryPointSuccess || !fn)
    return ABKV_ERR_CUDA;
  CUresult r = reinterpret_cast<EncodeTiled>(fn)(
      m, dtype, (cuuint32_t)rank, const_cast<void*>(base), dims, gstr, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
      swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ABKV_OK : ABKV_ERR_INVALID_ARG;
}

// 4D tensor map over bf16 with byte strides gstr (dims 1..3), 128B swizzle.
static inline int encode_tiled_4d(CUtensorMap* m, const void* base, const cuuint64_t (&dims)[4],
                                  const cuuint64_t (&gstr)[3], const cuuint32_t (&box)[4]) {
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, gstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace tc
}  // namespace abkv
