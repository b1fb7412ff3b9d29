// mxq_tp.cu -- the peer all-gather of the tensor-parallel decoder.
//
// Each rank of a sharded decoder owns whole output rows of every linear
// (output-feature sharding of mx_gemv, nn/tests/test_auto_generated.cpp:56:
// a row keeps its full K, so its block sums are those of the unsharded
// weight), so after each linear it holds some columns of the activation.
// One launch of tp_gather_kernel makes the full activation appear in every
// rank's mailbox: every thread stores its 16-byte pieces of this rank's
// columns into every rank's mailbox over NVLink (plain stores through CUDA
// IPC mappings), the grid's last CTA releases this rank's flag word in every
// mailbox, then waits, bounded, until every rank's flag in its own mailbox
// shows the same sequence number.  The kernel after it reads the gathered
// rows from the local mailbox once this grid has completed.
//
// Ordering: the copy starts after griddepcontrol.wait, so the producer's
// rows are complete; each CTA's stores are ordered before its arrival on the
// grid counter by a device fence, and the last CTA's system fence orders all
// of them before the release of the flags.  A slot (mailbox region) is
// reused only by the exchange after next: a rank can start that one only
// after every rank has joined the exchange in between, which every rank
// launches after the kernel that read the slot.
#include "mxq_internal.h"

namespace mxq {

namespace {

constexpr int kTpThreads = 256;

__global__ void __launch_bounds__(kTpThreads) tp_gather_kernel(TpGatherArgs a) {
  // the next kernel may start its prologue (weight streaming); it reads the
  // gathered rows only after its own griddepcontrol.wait, i.e. after this
  // grid has completed
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const long nth = (long)gridDim.x * kTpThreads;
  const long t0 = (long)blockIdx.x * kTpThreads + threadIdx.x;
  for (int s = 0; s < a.nseg; ++s) {
    const TpSegment g = a.seg[s];
    const size_t col = (size_t)a.rank * g.row_bytes;
    if (g.row_bytes % 16 == 0 && g.src_ld % 16 == 0 && g.dst_ld % 16 == 0 && g.dst_off % 16 == 0 &&
        (reinterpret_cast<uintptr_t>(g.src) & 15u) == 0) {
      const long per_row = (long)(g.row_bytes / 16), n = per_row * a.rows;
      for (long i = t0; i < n; i += nth) {
        const long r = i / per_row, c = i - r * per_row;
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(g.src + r * g.src_ld) + c);
        const size_t off = g.dst_off + (size_t)r * g.dst_ld + col + (size_t)c * 16;
        for (int p = 0; p < a.world; ++p) *reinterpret_cast<uint4*>(a.base[p] + off) = v;
      }
    } else {
      // ragged rows (the E8M0 scales of a slice): byte stores
      const long per_row = (long)g.row_bytes, n = per_row * a.rows;
      for (long i = t0; i < n; i += nth) {
        const long r = i / per_row, c = i - r * per_row;
        const uint8_t v = __ldcg(g.src + r * g.src_ld + c);
        const size_t off = g.dst_off + (size_t)r * g.dst_ld + col + (size_t)c;
        for (int p = 0; p < a.world; ++p) a.base[p][off] = v;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned old = atomicAdd(a.grid_cnt, 1u);
    if (old == gridDim.x - 1u) {
      *a.grid_cnt = 0u;
      const uint32_t next = *a.seq + 1u;
      if (a.world == 1) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        st_release_gpu(a.flag_out[0], next);
      } else {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int r = 0; r < a.world; ++r) st_release_sys(a.flag_out[r], next);
      }
      peer_wait(a.wait_flags, a.world, next, a.wait_ns ? a.wait_ns : kWaitLimitNs, a.status);
      *a.seq = next;
    }
  }
}

}  // namespace

cudaError_t launch_tp_gather(const TpGatherArgs& a, cudaStream_t st) {
  if (a.world < 1 || a.world > kMaxPeers || a.rank < 0 || a.rank >= a.world || a.rows < 1 || a.nseg < 1 ||
      a.nseg > 2 || !a.wait_flags || !a.seq || !a.grid_cnt)
    return cudaErrorInvalidValue;
  for (int r = 0; r < a.world; ++r)
    if (!a.base[r] || !a.flag_out[r]) return cudaErrorInvalidValue;
  long units = 0;
  for (int s = 0; s < a.nseg; ++s) {
    const TpSegment& g = a.seg[s];
    if (!g.src || g.row_bytes == 0 || g.src_ld < g.row_bytes || g.dst_ld < g.row_bytes * (size_t)a.world)
      return cudaErrorInvalidValue;
    units += (long)((g.row_bytes + 15) / 16) * a.rows;
  }
  // about one 16-byte piece per thread for a decode step's few kilobytes,
  // at most four CTAs per SM for a prompt chunk's megabytes
  long ctas = (units + kTpThreads - 1) / kTpThreads;
  if (ctas > 148L * 4) ctas = 148L * 4;
  if (ctas < 1) ctas = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kTpThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tp_gather_kernel, a);
}

}  // namespace mxq
