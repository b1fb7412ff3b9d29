// mxq_tp.cu -- peer exchanges over mailboxes: the partial sums of the
// tensor-parallel decoder and the expert outputs of the expert-parallel MoE.
//
// Each rank of a sharded decoder computes, for the O and down linears, a
// partial sum of every output row over its part of K (whole 32-blocks, so
// the MX block dots are those of the unsharded weight; the reference's
// mx_gemv sums them per row, nn/tests/test_auto_generated.cpp:56).  One
// launch of tp_gather_kernel makes every rank's partials appear in every
// rank's mailbox, [row][rank][values]: every thread stores its 16-byte
// pieces into every rank's mailbox over NVLink (plain stores through CUDA
// IPC mappings), the grid's last CTA releases this rank's flag word in every
// mailbox, then waits, bounded, until every rank's flag in its own mailbox
// shows the same sequence number.  The kernel after it (the residual) reads
// the partials from the local mailbox once this grid has completed and adds
// them in rank order.  The expert-parallel MoE uses the same launch to
// copy this rank's expert-output rows (a contiguous slot range) to the same
// rows of every other rank's mailbox.
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
  const long per_row = (long)(a.row_bytes / 16), n = per_row * a.rows;
  for (long i = (long)blockIdx.x * kTpThreads + threadIdx.x; i < n; i += nth) {
    const long r = i / per_row, c = i - r * per_row;
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(a.src) + i);
    const size_t off = a.dst_off + (size_t)r * a.row_stride + (size_t)a.rank * a.rank_stride + (size_t)c * 16;
    for (int p = 0; p < a.world; ++p)
      if (p != a.skip_rank) *reinterpret_cast<uint4*>(a.base[p] + off) = v;
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
  if (a.world < 1 || a.world > kMaxPeers || a.rank < 0 || a.rank >= a.world || a.rows < 0 ||
      (a.rows > 0 && (!a.src || a.row_bytes == 0 || a.row_bytes % 16 || a.dst_off % 16 || a.row_stride % 16 ||
                      a.rank_stride % 16 || (reinterpret_cast<uintptr_t>(a.src) & 15u))) ||
      !a.wait_flags || !a.seq || !a.grid_cnt)
    return cudaErrorInvalidValue;
  for (int r = 0; r < a.world; ++r)
    if (!a.base[r] || !a.flag_out[r] || (reinterpret_cast<uintptr_t>(a.base[r]) & 15u)) return cudaErrorInvalidValue;
  const long units = (long)(a.row_bytes / 16) * a.rows;
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
