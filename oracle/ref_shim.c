/* ref_shim.c - the one symbol the reference's CPU-only build is missing.
 *
 * TEST INFRASTRUCTURE ONLY. The reference's dsv4_matmul.c calls
 * dsv4_cuda_mmq_n (dsv4_matmul.c:572), but its stub (src/cuda/dsv4_cuda_stub.c)
 * does not define it, so a CPU-only link fails. With the stub,
 * dsv4_cuda_has() is always 0 and this is unreachable. */
#include <stddef.h>
struct DSV4QMat_;
void dsv4_cuda_mmq_n(float *y, const float *x, const void *m, int nt)
{
    (void)y; (void)x; (void)m; (void)nt;
}
