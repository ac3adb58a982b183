// IQ2_XXS / IQ2_XS / IQ2_S / IQ3_XXS / IQ3_S lattice-search kernels (sm_100a).
#include "qs_kernels.h"

namespace qs {

struct IqTables {
    int dummy;
};

cudaError_t iq_tables_create(IqTables** out) {
    *out = new IqTables{0};
    return cudaSuccess;
}

void iq_tables_destroy(IqTables* t) { delete t; }

cudaError_t launch_iq(int, const QuantArgs&, const LaunchCtx&, const IqTables*) { return cudaErrorNotSupported; }

}  // namespace qs
