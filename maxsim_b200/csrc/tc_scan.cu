// Tensor-core (tcgen05) scan engine -- placeholder until the sm_100a kernel lands.
#include "common.cuh"

namespace msb {
bool tc_scan_supported(const DocsView&, const QueryView&, const ReduceView&, const TargetsView&, bool) { return false; }
size_t tc_scan_workspace_bytes(const DocsView&, const QueryView&, const TargetsView&) { return 0; }
void launch_tc_scan(const DocsView&, const QueryView&, const ReduceView&, const TargetsView&, float*, void*, size_t,
                    cudaStream_t) {
  throw NotSupported("tensor-core scan engine not built");
}
}  // namespace msb
