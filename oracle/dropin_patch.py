"""TEST INFRASTRUCTURE -- the drop-in proof: write a copy of the reference's
tinylm.c with libtinylm_cuda at its five seams.

    python oracle/dropin_patch.py <reference tinylm.c> <output .c>

Run by `make -C oracle dropin` at build time; the copy goes to
oracle/_ref/cuda/tinylm.c (git-ignored, never committed) and is compiled with
-DUSE_CUDA into the reference's own CLI (oracle/_ref/tinylm_cuda) and into the
reference-leg harness (oracle/_ref/libtlref_cuda.so).

The patch is the one INTEGRATION.md documents, and nothing else:
  * after the includes: the USE_CUDA header block (tinylm_cuda.h, a status
    check that exits as the reference does on fatal errors, and a one-time set-up:
    tl_init on TL_DEVICE (default 0) + tl_set_host_buffers(1), so the library
    takes the reference's own calloc'd buffers);
  * first statement of mm (tinylm.c:439), mm_bt (480), mm_atb (510), adamw
    (1159) and global_gradnorm (1171): an `#ifdef USE_CUDA` block that calls
    tl_matmul / tl_matmul_bt / tl_matmul_at / tl_adamw_step / tl_grad_norm
    with the function's own arguments and returns.
Without -DUSE_CUDA the copy compiles to the reference unchanged.  Each anchor
must match exactly once, or the script fails.
"""
import re
import sys

HEADER = r'''
#ifdef USE_CUDA
/* ---- libtinylm_cuda seams (B200 drop-in build) ----------------------------
 * The primitives below call the library with the reference's own host
 * buffers; host-buffer mode stages them through GPU memory and each call
 * returns with its result in host memory.  Errors end the process, as the
 * reference's own fatal errors do. */
#include "tinylm_cuda.h"
static void tl_seam_check(int rc, const char *what){
    if(rc){ fprintf(stderr, "libtinylm_cuda: %s: %s\n", what, tl_last_error()); exit(1); }
}
static void tl_seam_init(void){
    static int ready = 0;
    if(ready) return;
    const char *d = getenv("TL_DEVICE");
    tl_seam_check(tl_init(d ? atoi(d) : 0), "tl_init");
    tl_seam_check(tl_set_host_buffers(1), "tl_set_host_buffers");
    ready = 1;
}
#define TL_SEAM(call) do { tl_seam_init(); tl_seam_check((call), #call); } while (0)
#endif
'''

SEAMS = [
    (r"static void mm\([^)]*\)\s*\{",
     "    TL_SEAM(tl_matmul(Y, X, W, M, K, N)); return;"),
    (r"static void mm_bt\([^)]*\)\s*\{",
     "    TL_SEAM(tl_matmul_bt(dX, dY, W, M, K, N)); return;"),
    (r"static void mm_atb\([^)]*\)\s*\{",
     "    TL_SEAM(tl_matmul_at(dW, X, dY, M, K, N)); return;"),
    (r"static void adamw\([^)]*\)\s*\{",
     "    TL_SEAM(tl_adamw_step(P, G, M, Vv, n, lr, b1, b2, wd, t, gscale)); return;"),
    (r"static float global_gradnorm\([^)]*\)\s*\{",
     "    { float nrm = 0.0f; TL_SEAM(tl_grad_norm(G, n, &nrm)); return nrm; }"),
]


def patch(src):
    m = list(re.finditer(r"^#include <immintrin.h>[^\n]*\n", src, flags=re.M))
    if len(m) != 1:
        raise SystemExit("dropin_patch: include anchor not found exactly once")
    src = src[:m[0].end()] + HEADER + src[m[0].end():]
    for pat, call in SEAMS:
        m = list(re.finditer(pat, src))
        if len(m) != 1:
            raise SystemExit(f"dropin_patch: anchor {pat!r} matched {len(m)} times")
        block = "\n#ifdef USE_CUDA\n" + call + "\n#endif\n"
        src = src[:m[0].end()] + block + src[m[0].end():]
    return src


def main(argv):
    if len(argv) != 3:
        raise SystemExit(__doc__)
    with open(argv[1]) as f:
        src = f.read()
    with open(argv[2], "w") as f:
        f.write(patch(src))


if __name__ == "__main__":
    main(sys.argv)
