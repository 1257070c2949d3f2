// Host side of the tensor-core chunked path: buffer layouts, tensor maps and the two orchestrations.
#include "gdn_chunk_impl.cuh"

namespace qbgdn {

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

// [rows, heads, dim] bf16 activations; box = 64 columns x 1 head x 64 rows, 128-byte swizzle.
bool map_act(CUtensorMap* m, const void* base, int64_t rows, int heads, int dim, int box_rows = 64) {
  EncodeTiled f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)dim * 2, (cuuint64_t)heads * dim * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
  cuuint32_t es[3] = {1, 1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 rows [rows, heads, dim] read as boxes of box_cols x box_rows of one head (the value or
// output-gradient rows of a chunk), unswizzled or (sw64) in the 64-byte swizzle of an MN-major MMA
// operand with 64-byte rows; rows past the end read as zero.
bool map_rows(CUtensorMap* m, const void* base, int64_t rows, int heads, int dim, int box_cols, int box_rows,
              bool f32 = false, bool sw64 = false) {
  EncodeTiled f = encode_fn();
  if (!f) return false;
  const cuuint64_t eb = f32 ? 4 : 2;
  cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)dim * eb, (cuuint64_t)heads * dim * eb};
  cuuint32_t box[3] = {(cuuint32_t)box_cols, 1, (cuuint32_t)box_rows};
  cuuint32_t es[3] = {1, 1, 1};
  return f(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
           dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, sw64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// State rows [rows, 128] fp32 (a chunk-state buffer); box = 32 columns x 32 rows in the 32-byte-atom
// swizzle: four boxes make the MN-major tf32 operand of a 32-row slice.
bool map_state_mn(CUtensorMap* m, const void* base, int64_t rows) {
  EncodeTiled f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {128, (cuuint64_t)rows};
  cuuint64_t strides[1] = {128 * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t es[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t a256(int64_t x) { return (x + 255) & ~int64_t(255); }

// The chunk intermediates: [ckpt][gates] fp32, the forward's T, P and [K; Q] operand images and its
// tf32-rounded D tiles.
struct Saved {
  float *ckpt, *gates;
  uint8_t *Timg, *Pimg, *KQimg;
  float* Ds;
};

// with_ckpt false: the layout without its chunk-start states (a backward given them by the caller).
int64_t saved_layout(int Hv, int Hk, int64_t n_chunks, char* base, Saved* s, bool with_ckpt = true) {
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* at = base ? base + off : nullptr;
    off += a256(bytes);
    return at;
  };
  Saved x;
  x.ckpt = (float*)take(with_ckpt ? n_chunks * Hv * (int64_t)DV * DK * 4 : 0);
  x.gates = (float*)take(n_chunks * Hv * 128 * 4);
  x.Timg = (uint8_t*)take(n_chunks * Hv * 16384);
  x.Pimg = (uint8_t*)take(n_chunks * Hv * 16384);
  x.KQimg = (uint8_t*)take(n_chunks * Hk * 32768);
  x.Ds = (float*)take(n_chunks * Hv * 64 * DV * 4);
  if (s) *s = x;
  return off;
}

// Workspace: [status block][chunk_off][fwd: T, P and [K; Q] images, gates when nothing is saved | bwd:
// dS per chunk, the [dO; F] images, per-chunk head sums (layer mode), and a saved buffer plus forward
// workspace when the backward recomputes].  The status block opens the workspace (qb_gdn_status reads
// it there); a nested forward workspace keeps one of its own, unused (the recompute reports into the
// backward's).
struct Ws {
  int* err;          // the status block (status.cuh), initialised by each call
  int64_t* chunk_off;
  uint8_t *Timg, *Pimg, *KQimg;
  float* gates;
  float* dsbuf;
  uint8_t* Aimg;     // [dO; F] operand images from the reverse walk, [chunks, Hv, 4] x 16 KB
  float* head_part;
  char* saved;
  char* fwd_ws;
};

int64_t ws_layout(int Hv, int Hk, int N, int64_t n_chunks, bool layer, bool varlen, int op, bool with_saved,
                  char* base, Ws* w, bool ckpt_external = false) {
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* at = base ? base + off : nullptr;
    off += a256(bytes);
    return at;
  };
  Ws x{};
  x.err = (int*)take(kStatusBytes);
  x.chunk_off = (int64_t*)take(varlen ? (int64_t)(N + 1) * 8 : 0);
  if (op == 0) {
    x.Timg = (uint8_t*)take(n_chunks * Hv * 16384);
    x.Pimg = (uint8_t*)take(n_chunks * Hv * 16384);
    x.KQimg = (uint8_t*)take(n_chunks * Hk * 32768);
    x.gates = (float*)take(n_chunks * Hv * 128 * 4);
  } else {
    x.dsbuf = (float*)take(n_chunks * Hv * (int64_t)DV * DK * 4);
    x.Aimg = (uint8_t*)take(n_chunks * Hv * (DV / DVT) * 16384);
    x.head_part = (float*)take(layer ? n_chunks * Hv * 2 * 4 : 0);
    if (with_saved) {
      x.saved = take(saved_layout(Hv, Hk, n_chunks, nullptr, nullptr, !ckpt_external));
      x.fwd_ws = take(ws_layout(Hv, Hk, N, n_chunks, layer, varlen, 0, false, nullptr, nullptr));
    }
  }
  if (w) *w = x;
  return off;
}

}  // namespace

bool chunked_supported(int Dk, int Dv) { return Dk == DK && Dv == DV && encode_fn() != nullptr; }
bool chunked_bwd_ready() { return true; }

int64_t chunked_saved_bytes(int Hv, int Hk, int64_t n_chunks, int64_t tokens, bool layer) {
  return saved_layout(Hv, Hk, n_chunks, nullptr, nullptr);
}

int64_t chunked_ws_bytes(int Hv, int Hk, int N, int64_t n_chunks, int64_t tokens, bool varlen, int op, bool with_saved,
                         bool layer, bool ckpt_external) {
  return ws_layout(Hv, Hk, N, n_chunks, layer, varlen, op, with_saved, nullptr, nullptr, ckpt_external);
}

cudaError_t chunked_fwd(const ChunkFwdArgs& a, void* ws, cudaStream_t st, int* status) {
  if (!a.in_bf16) return cudaErrorInvalidValue;
  const bool layer = a.g == nullptr;
  const int64_t rows = (int64_t)a.B * a.T;
  Ws w;
  ws_layout(a.Hv, a.Hk, a.N, a.n_chunks, layer, a.cu != nullptr, 0, false, (char*)ws, &w);
  Saved sv{};
  float *gates = w.gates, *ckpt = nullptr;
  uint8_t *Ti = w.Timg, *Pi = w.Pimg, *KQi = w.KQimg;
  if (a.saved) {
    saved_layout(a.Hv, a.Hk, a.n_chunks, (char*)a.saved, &sv, a.ckpt_in == nullptr);
    gates = sv.gates, ckpt = a.ckpt_in ? nullptr : sv.ckpt;
    Ti = sv.Timg, Pi = sv.Pimg, KQi = sv.KQimg;
  }
  cudaError_t e;
  int* err = status;  // initialised by the caller (a recomputing backward passes its own)
  if (a.cu && (e = launch_chunk_offsets(a.cu, a.N, w.chunk_off, st)) != cudaSuccess) return e;
  CUtensorMap kmap, qmap;
  if (!map_act(&kmap, a.k, rows, a.Hk, a.Dk) || !map_act(&qmap, a.q, rows, a.Hk, a.Dk)) return cudaErrorInvalidValue;
  Geo geo{a.T, a.Hk, a.Hv, a.N, (a.T + C - 1) / C, a.cu, a.cu ? w.chunk_off : nullptr};
  if (a.n_chunks > 0) {
    PrepArgs pa{geo, a.g, a.beta, a.a_raw, a.b_raw, a.A_log, a.dt_bias, Ti, Pi, KQi, gates, err};
    if ((e = launch_chunk_prep(kmap, qmap, pa, a.n_chunks, a.Hk, st)) != cudaSuccess) return e;
  }
  CUtensorMap vmap, ymap;
  // (bf16 tiles of 64-byte rows in the 64-byte swizzle: the walk's row reads and writes spread over the banks)
  if (!map_rows(&vmap, a.v, rows, a.Hv, a.Dv, DVT, C, false, true) ||
      !map_rows(&ymap, a.y, rows, a.Hv, a.Dv, DVT, C, !a.out_bf16, a.out_bf16))
    return cudaErrorInvalidValue;
  StateArgs sa{geo, a.v, gates, a.h0, a.y, a.hT, ckpt, Ti, Pi, KQi, a.saved ? sv.Ds : nullptr, err, a.ckpt_in,
               a.n_chunks};
  if (a.ckpt_in && (a.n_chunks == 0 || a.hT)) return cudaErrorInvalidValue;  // recompute mode writes D alone
  return launch_chunk_fwd_state(vmap, ymap, sa, a.Hv, a.N, a.out_bf16, st);
}

cudaError_t chunked_bwd(const ChunkBwdArgs& a, void* ws, cudaStream_t st) {
  if (!a.in_bf16) return cudaErrorInvalidValue;
  const bool layer = a.g == nullptr;
  const int64_t rows = (int64_t)a.B * a.T;
  Ws w;
  ws_layout(a.Hv, a.Hk, a.N, a.n_chunks, layer, a.cu != nullptr, 1, a.saved == nullptr, (char*)ws, &w,
            a.ckpt_in != nullptr);
  cudaError_t e;
  const void* saved = a.saved;
  if (!saved) {  // recompute the forward's intermediates with the same forward (y is discarded into dv)
    ChunkFwdArgs f{};
    f.B = a.B, f.T = a.T, f.Hk = a.Hk, f.Hv = a.Hv, f.Dk = a.Dk, f.Dv = a.Dv, f.N = a.N, f.n_chunks = a.n_chunks;
    f.cu = a.cu, f.q = a.q, f.k = a.k, f.v = a.v, f.g = a.g, f.beta = a.beta, f.h0 = a.h0, f.y = a.dv;
    f.saved = w.saved, f.in_bf16 = a.in_bf16, f.out_bf16 = a.out_bf16;
    f.a_raw = a.a_raw, f.b_raw = a.b_raw, f.A_log = a.A_log, f.dt_bias = a.dt_bias;
    f.ckpt_in = a.ckpt_in;  // given the chunk-start states: every chunk recomputed on its own (no walk)
    if (a.n_chunks > 0 && (e = chunked_fwd(f, w.fwd_ws, st, w.err)) != cudaSuccess) return e;
    saved = w.saved;
  }
  Saved sv;
  saved_layout(a.Hv, a.Hk, a.n_chunks, (char*)saved, &sv, a.ckpt_in == nullptr);
  if (a.ckpt_in) sv.ckpt = const_cast<float*>(a.ckpt_in);
  if (a.cu && (e = launch_chunk_offsets(a.cu, a.N, w.chunk_off, st)) != cudaSuccess) return e;
  Geo geo{a.T, a.Hk, a.Hv, a.N, (a.T + C - 1) / C, a.cu, a.cu ? w.chunk_off : nullptr};
  CUtensorMap dmap, vmap, dvmap;
  if (!map_rows(&dmap, a.dy, rows, a.Hv, a.Dv, DVT, C, false, true) ||
      !map_rows(&vmap, a.v, rows, a.Hv, a.Dv, DVT, C, false, true) ||
      !map_rows(&dvmap, a.dv, rows, a.Hv, a.Dv, DVT, C, !a.out_bf16, a.out_bf16))
    return cudaErrorInvalidValue;
  BwdStateArgs ba{geo, a.dy, sv.gates, a.dhT, a.dv, a.dh0, w.dsbuf, sv.Timg, sv.Pimg, sv.KQimg, w.Aimg, w.err};
  if ((e = launch_chunk_bwd_state(dmap, dvmap, ba, a.Hv, a.N, a.out_bf16, st)) != cudaSuccess) return e;
  if (a.n_chunks == 0) {
    if (layer) {
      if ((e = cudaMemsetAsync(a.dA_log, 0, a.Hv * 4, st)) != cudaSuccess) return e;
      if ((e = cudaMemsetAsync(a.ddt_bias, 0, a.Hv * 4, st)) != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  CUtensorMap smap_mn, dmap_mn;
  if (!map_state_mn(&smap_mn, sv.ckpt, a.n_chunks * a.Hv * (int64_t)DV) ||
      !map_state_mn(&dmap_mn, w.dsbuf, a.n_chunks * a.Hv * (int64_t)DV))
    return cudaErrorInvalidValue;
  GradArgs ga{geo, a.g, sv.gates, sv.KQimg, sv.Ds, w.Aimg, a.dq, a.dk, a.dg, a.dbeta, w.err,
              static_cast<const __nv_bfloat16*>(a.q), static_cast<const __nv_bfloat16*>(a.k),
              a.a_raw, a.b_raw, a.A_log, a.dt_bias, w.head_part, a.dA_log, a.ddt_bias,
              reinterpret_cast<unsigned*>(w.err + 2)};
  // the tiles of full chunks' dq, dk rows (bf16 results; a float32 result is stored row by row and the
  // maps are not read)
  CUtensorMap dqmap = vmap, dkmap = vmap;
  if (a.out_bf16 && (!map_act(&dqmap, a.dq, rows, a.Hk, a.Dk) || !map_act(&dkmap, a.dk, rows, a.Hk, a.Dk)))
    return cudaErrorInvalidValue;
  return launch_chunk_bwd_grad(smap_mn, dmap_mn, vmap, dqmap, dkmap, ga, a.n_chunks, a.Hk, a.out_bf16, st);
}

}  // namespace qbgdn
