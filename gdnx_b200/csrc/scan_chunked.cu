// Chunked WY/UT tensor-core scan -- placeholder until the tcgen05 kernel lands.
#include "kernels.h"

namespace gdnx {

bool chunked_eligible(const gdnx_scan_args&) { return false; }
size_t chunked_workspace_bytes(const gdnx_scan_args&) { return 0; }
gdnx_status launch_chunked_scan(const gdnx_scan_args&, cudaStream_t) { return GDNX_EUNSUPPORTED; }

}  // namespace gdnx
