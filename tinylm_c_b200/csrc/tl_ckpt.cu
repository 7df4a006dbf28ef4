// tl_ckpt.cu -- host-side pieces of the training loop: the reference's
// checkpoint formats, its learning-rate schedule and its batch sampler.
//
//   TLM4 bundle  (model_save_bundle, tinylm.c:1895-1914): "TLM4", 11 int32
//                header {V,D,L,H,KV,F,T,eot,tmpl,n_mtp,n_exp}, n fp32
//                parameters (map_weights order), int32 tokenizer length, blob.
//                Loading also accepts TLM1-TLM3 headers (hdr_ints, 1691-1700).
//   TOPT sidecar (opt_save/opt_load, 2526-2539): "TOPT", int32 iter, M[n], V[n].
//                Written and read by ranges, so each ZeRO-1 rank stores and
//                restores its own shard of M and V without any gather.
//   LR schedule  (train_loop 2587-2590): linear warm-up, then cosine to 0.1*lr.
//   Sampler      (train_loop 2596-2626): xorshift64 window starts into a
//                uint16 token stream, targets shifted by one (and by 2+k for
//                the MTP heads).
// Buffers passed here may be host or device memory; device data is staged
// through a bounded host buffer.  All functions are host-only.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>
#include "tl_common.cuh"

namespace tl {

static bool is_device(const void *p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice;
}

constexpr size_t kStageFloats = 4u << 20;  // 16 MiB host staging for device data

// fwrite n floats from host or device memory.
static int write_floats(FILE *f, const float *src, size_t n, const char *what) {
  if (n == 0) return TL_OK;
  if (!is_device(src)) {
    if (fwrite(src, sizeof(float), n, f) != n) return set_error(TL_EINVAL, "write failed (%s)", what);
    return TL_OK;
  }
  std::vector<float> buf(std::min(n, kStageFloats));
  for (size_t o = 0; o < n; o += buf.size()) {
    const size_t k = std::min(buf.size(), n - o);
    cudaError_t e = cudaMemcpy(buf.data(), src + o, k * sizeof(float), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_check(e, "cudaMemcpy(checkpoint read-back)");
    if (fwrite(buf.data(), sizeof(float), k, f) != k) return set_error(TL_EINVAL, "write failed (%s)", what);
  }
  return TL_OK;
}

// fread n floats into host or device memory.
static int read_floats(FILE *f, float *dst, size_t n, const char *what) {
  if (n == 0) return TL_OK;
  if (!is_device(dst)) {
    if (fread(dst, sizeof(float), n, f) != n) return set_error(TL_EINVAL, "file too short (%s)", what);
    return TL_OK;
  }
  std::vector<float> buf(std::min(n, kStageFloats));
  for (size_t o = 0; o < n; o += buf.size()) {
    const size_t k = std::min(buf.size(), n - o);
    if (fread(buf.data(), sizeof(float), k, f) != k) return set_error(TL_EINVAL, "file too short (%s)", what);
    cudaError_t e = cudaMemcpy(dst + o, buf.data(), k * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_check(e, "cudaMemcpy(checkpoint upload)");
  }
  return TL_OK;
}

}  // namespace tl

using namespace tl;

TL_API int tl_ckpt_save_bundle(const char *path, const int *hdr11, const float *P, size_t n, const void *tok_blob,
                               int tok_len) {
  if (!path || !hdr11 || (!P && n)) return set_error(TL_EINVAL, "NULL argument");
  FILE *f = fopen(path, "wb");
  if (!f) return set_error(TL_EINVAL, "cannot write %s", path);
  int rc = TL_OK;
  if (fwrite("TLM4", 1, 4, f) != 4 || fwrite(hdr11, 4, 11, f) != 11) rc = set_error(TL_EINVAL, "write failed");
  if (!rc) rc = write_floats(f, P, n, "parameters");
  const int tl = tok_blob ? tok_len : 0;
  if (!rc && fwrite(&tl, 4, 1, f) != 1) rc = set_error(TL_EINVAL, "write failed");
  if (!rc && tl > 0 && fwrite(tok_blob, 1, (size_t)tl, f) != (size_t)tl) rc = set_error(TL_EINVAL, "write failed");
  if (fclose(f) != 0 && !rc) rc = set_error(TL_EINVAL, "close failed for %s", path);
  return rc;
}

// Reads the header (hdr11 gets V,D,L,H,KV,F,T,eot,tmpl,n_mtp,n_exp; fields the
// file's version lacks are 0) and, when P is not NULL, the n_expected
// parameters.  *n_in_file receives the number of 4-byte words after the
// header: the parameter block plus the int32 tokenizer length and the
// tokenizer blob, so it is an upper bound on the parameter count (a bundle of
// n parameters has *n_in_file >= n + 1), not the count itself.
TL_API int tl_ckpt_load_bundle(const char *path, int *hdr11, float *P, size_t n_expected, size_t *n_in_file) {
  if (!path || !hdr11) return set_error(TL_EINVAL, "NULL argument");
  FILE *f = fopen(path, "rb");
  if (!f) return set_error(TL_EINVAL, "cannot open %s", path);
  char m[4];
  int nh = 0;
  if (fread(m, 1, 4, f) == 4) {
    if (!memcmp(m, "TLM4", 4)) nh = 11;
    else if (!memcmp(m, "TLM3", 4)) nh = 10;
    else if (!memcmp(m, "TLM2", 4)) nh = 9;
    else if (!memcmp(m, "TLM1", 4)) nh = 8;
  }
  if (!nh) {
    fclose(f);
    return set_error(TL_EINVAL, "%s: not a TLM1-TLM4 bundle (windowed, QK-norm, shared-expert and quantized "
                     "formats are outside this training path)", path);
  }
  int h[11] = {0};
  if (fread(h, 4, (size_t)nh, f) != (size_t)nh) {
    fclose(f);
    return set_error(TL_EINVAL, "%s: truncated header", path);
  }
  memcpy(hdr11, h, sizeof(h));
  long here = ftell(f);
  fseek(f, 0, SEEK_END);
  long end = ftell(f);
  fseek(f, here, SEEK_SET);
  if (n_in_file) *n_in_file = (size_t)(end - here) / 4;
  int rc = TL_OK;
  if (P && (size_t)(end - here) < n_expected * 4 + 4)
    rc = set_error(TL_EINVAL, "%s holds fewer than the %zu expected parameters and the tokenizer length", path,
                   n_expected);
  if (P && !rc) rc = read_floats(f, P, n_expected, "parameters");
  fclose(f);
  return rc;
}

TL_API int tl_ckpt_opt_create(const char *path, int iter, size_t n) {
  if (!path) return set_error(TL_EINVAL, "NULL path");
  FILE *f = fopen(path, "wb");
  if (!f) return set_error(TL_EINVAL, "cannot write %s", path);
  int rc = TL_OK;
  if (fwrite("TOPT", 1, 4, f) != 4 || fwrite(&iter, 4, 1, f) != 1) rc = set_error(TL_EINVAL, "write failed");
  // size the file: M[n] and V[n] follow; ranges are filled by tl_ckpt_opt_write
  if (!rc && n > 0) {
    if (fseek(f, (long)(8 + 2 * n * sizeof(float)) - 1, SEEK_SET) != 0 || fputc(0, f) == EOF)
      rc = set_error(TL_EINVAL, "cannot size %s", path);
  }
  if (fclose(f) != 0 && !rc) rc = set_error(TL_EINVAL, "close failed for %s", path);
  return rc;
}

// M[offset, offset+count) and V[offset, offset+count) of a TOPT file of n floats each.
TL_API int tl_ckpt_opt_write(const char *path, size_t n, size_t offset, const float *M, const float *V, size_t count) {
  if (!path || (!M && count) || (!V && count)) return set_error(TL_EINVAL, "NULL argument");
  if (offset > n || count > n - offset) return set_error(TL_EINVAL, "range [%zu, +%zu) outside %zu", offset, count, n);
  FILE *f = fopen(path, "r+b");
  if (!f) return set_error(TL_EINVAL, "cannot open %s (create it with tl_ckpt_opt_create)", path);
  int rc = TL_OK;
  if (fseek(f, (long)(8 + offset * sizeof(float)), SEEK_SET) != 0) rc = set_error(TL_EINVAL, "seek failed");
  if (!rc) rc = write_floats(f, M, count, "M");
  if (!rc && fseek(f, (long)(8 + (n + offset) * sizeof(float)), SEEK_SET) != 0) rc = set_error(TL_EINVAL, "seek failed");
  if (!rc) rc = write_floats(f, V, count, "V");
  if (fclose(f) != 0 && !rc) rc = set_error(TL_EINVAL, "close failed for %s", path);
  return rc;
}

TL_API int tl_ckpt_opt_read(const char *path, size_t n, size_t offset, float *M, float *V, size_t count,
                            int *iter_out) {
  if (!path) return set_error(TL_EINVAL, "NULL path");
  if (offset > n || count > n - offset) return set_error(TL_EINVAL, "range [%zu, +%zu) outside %zu", offset, count, n);
  FILE *f = fopen(path, "rb");
  if (!f) return set_error(TL_EINVAL, "cannot open %s", path);
  char m[4];
  int iter = 0, rc = TL_OK;
  if (fread(m, 1, 4, f) != 4 || memcmp(m, "TOPT", 4) || fread(&iter, 4, 1, f) != 1)
    rc = set_error(TL_EINVAL, "%s: not a TOPT file", path);
  if (!rc && count) {
    if (fseek(f, (long)(8 + offset * sizeof(float)), SEEK_SET) != 0) rc = set_error(TL_EINVAL, "seek failed");
    if (!rc) rc = read_floats(f, M, count, "M");
    if (!rc && fseek(f, (long)(8 + (n + offset) * sizeof(float)), SEEK_SET) != 0) rc = set_error(TL_EINVAL, "seek failed");
    if (!rc) rc = read_floats(f, V, count, "V");
  }
  fclose(f);
  if (!rc && iter_out) *iter_out = iter;
  return rc;
}

// Learning rate at iteration `it` (train_loop, tinylm.c:2587-2590): linear
// warm-up over `warmup` iterations, then a cosine from lr down to 0.1*lr.
TL_API float tl_lr_at(int it, float lr, int iters, float warmup) {
  if (it < warmup) return lr * (it + 1) / warmup;
  float r = (it - warmup) / (float)(iters > warmup ? iters - warmup : 1);
  if (r > 1) r = 1;
  return 0.1f * lr + 0.5f * (1 + cosf(3.14159265f * r)) * (lr - 0.1f * lr);
}

static inline uint64_t xorshift64(uint64_t *s) {
  uint64_t x = *s;
  x ^= x << 13; x ^= x >> 7; x ^= x << 17;
  *s = x;
  return x;
}

// B windows of a uint16 stream, drawn with the reference's generator state
// *rng.  Training batches (val = 0, tinylm.c:2623-2626): start = rng % (n -
// (T + n_mtp + 2)), tok = s[start+j], tgt = s[start+j+1], tgt_mtp[k] =
// s[start+j+2+k] (k-major, [n_mtp][B*T]).  Validation batches (val = 1,
// 2596-2597): start = rng % (n - T - 1), no MTP targets.
TL_API int tl_sample_windows(unsigned long long *rng, const unsigned short *stream, size_t n, int B, int T,
                             int n_mtp, int val, int *tok, int *tgt, int *tgt_mtp) {
  if (!rng || !stream || !tok || !tgt || B < 0 || T < 1) return set_error(TL_EINVAL, "bad argument");
  const size_t span = val ? (size_t)T + 1 : (size_t)T + n_mtp + 2;
  if (n <= span) return set_error(TL_EINVAL, "token stream of %zu is too short for windows of %zu", n, span);
  const int nm = val ? 0 : n_mtp;
  if (nm > 0 && !tgt_mtp) return set_error(TL_EINVAL, "tgt_mtp is NULL");
  uint64_t s = *rng;
  const size_t N = (size_t)B * T;
  for (int i = 0; i < B; i++) {
    const size_t st = (size_t)(xorshift64(&s) % (uint64_t)(n - span));
    for (int j = 0; j < T; j++) {
      const size_t r = (size_t)i * T + j;
      tok[r] = stream[st + j];
      tgt[r] = stream[st + j + 1];
      for (int k = 0; k < nm; k++) tgt_mtp[(size_t)k * N + r] = stream[st + j + 2 + k];
    }
  }
  *rng = s;
  return TL_OK;
}
