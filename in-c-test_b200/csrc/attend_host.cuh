// attend_host.cuh -- host-side types of the decode attend path.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "attend_common.cuh"

namespace kvl {

// One sequence whose output is combined from `count` partials; part p is
// stored at part index first + p * step.
struct MergeEntry {
  int seq;
  int first;
  int count;
  int step;
};

// Stream-K decomposition of a batch (host copy).
struct HostPlan {
  int batch = 0;
  int grid = 0;
  int nparts = 0;
  std::vector<AttendSegment> segs;
  std::vector<int> cta_seg;          // grid + 1
  std::vector<long long> seq_row0;   // batch
  std::vector<int> seq_len;          // batch
  std::vector<MergeEntry> merges;
  int max_merge_count = 0;
};

int build_attend_plan(HostPlan &hp, int batch, const int *seq_len, const long long *seq_row0,
                      int max_ctas);
int build_concat_plan(HostPlan &hp, int count, const int *seq_len, const long long *seq_row0, int max_ctas);

struct AttendLaunch {
  bool q8 = false;
  int nh = kHeads, R = kLatent, DR = kRope;
  long long rows = 0;
  const float *q = nullptr;
  float *out = nullptr;
  float *lse = nullptr;
  const uint16_t *kv = nullptr;       // bf16 pool [rows][R + DR]
  const float *kvf = nullptr;         // fp32 rows [rows][R + DR], read instead of kv by the
                                      // CUDA-core kernel (shapes other than 16 x 512 x 64)
  const int8_t *lat8 = nullptr;       // q8 pool [rows][R]
  const float *lscale = nullptr;      // q8 pool [rows]
  const uint16_t *rope16 = nullptr;   // q8 pool [rows][DR]
  float softmax_scale = 0.f;
  bool skip_merge = false;            // leave split sequences as partials (a cross-GPU combine reads them)
  // the previous kernel on the stream writes q and was launched as a
  // programmatic dependent that releases its own dependents only after its
  // wait (the decode step's absorb kernels): the attend may start during it
  bool q_dependent = false;
};

// Device-resident copy of a plan plus the partial-output workspace.
struct DevicePlan {
  HostPlan host;
  void *d_meta = nullptr;
  size_t meta_bytes = 0;
  void *d_work = nullptr;
  size_t work_bytes = 0;
  size_t off_segs = 0, off_cta = 0, off_row0 = 0, off_merge = 0, off_len = 0, off_err = 0;
  float *part_o = nullptr;
  float *part_lse = nullptr;
  uint8_t *qimg = nullptr;  // [batch][kQImgStride] query images

  int upload(const HostPlan &hp, int nh, int R, cudaStream_t stream, void *pinned, size_t pinned_bytes);
  int launch(const AttendLaunch &a, cudaStream_t stream) const;
  uint32_t *err_word() const;
  void release();
};

bool make_tmap_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t inner,
                  uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                  CUtensorMapSwizzle sw);

cudaError_t launch_merge(float *out, float *lse, const float *part_o, const float *part_lse,
                         const MergeEntry *d_entries, int n_entries, int nh, int R,
                         cudaStream_t stream, int max_count);
cudaError_t launch_merge_packed(float *out, float *lse, const float *parts_base, int parts, int batch, int nh,
                                int R, cudaStream_t stream);

}  // namespace kvl
