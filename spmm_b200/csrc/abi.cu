// abi.cu -- status text and ABI version of the spmm_b200 C interface.
#include <atomic>

#include "../../include/spmm_b200.h"
#include "common.cuh"

extern "C" const char *spmm_status_string(int status) {
    switch (status) {
        case SPMM_OK: return "ok";
        case SPMM_EINVAL: return "invalid argument";
        case SPMM_ELABEL: return "cluster label out of range";
        case SPMM_EOVERFLOW_U16:
            return "csr_to_boo: block local index space exceeds uint16 -- reduce max_nr/max_nc in "
                   "the clustering";
        case SPMM_EDUPLICATE: return "csr_to_pbr: duplicate (row, col) entries in the input CSR";
        case SPMM_ECUDA: return "CUDA error";
        case SPMM_EWORKSPACE: return "workspace too small";
        case SPMM_EUNSUPPORTED: return "size or type not supported";
        case SPMM_EALIGN: return "misaligned pointer";
        case SPMM_ESCRATCH:
            return "spmm_boo_build_noalloc: problem exceeds the 32 MiB static scratch";
        case SPMM_ETIMEOUT:
            return "a bounded device wait expired: the product stopped early and Y is incomplete";
        case SPMM_ENCCL: return "a collective (NCCL / process group) failed or timed out";
        default: return "unknown status";
    }
}

extern "C" int spmm_abi_version(void) { return 2; }

namespace spmm {
static std::atomic<uint64_t> g_product_launches{0};
void note_product_launch() { g_product_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace spmm

extern "C" uint64_t spmm_product_launches(void) { return spmm::g_product_launches.load(std::memory_order_relaxed); }
