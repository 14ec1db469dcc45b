// bt_elem.cuh -- the element type of one compilation of the value-facing kernels.
//
// No include guard: bt_body.cuh includes it inside each element namespace.  IEEE binary16 by
// default; bfloat16 when BT_ELEM_BF16 is defined.  Both are 16-bit sign-magnitude formats, so
// one descending key codec serves both (reference: include/type_codec.cuh:13-38 for fp16);
// only the exponent field (which sets the NaN test and -inf), the NaN used as a fill value
// and the paired hardware type differ.

#ifdef BT_ELEM_BF16
using h2t = __nv_bfloat162;
constexpr uint32_t kExpBits = 0x7F80u;   // exponent field; above it (sign cleared): NaN
constexpr uint32_t kNaN2 = 0x7FC07FC0u;  // a quiet NaN in both halves
#else
using h2t = __half2;
constexpr uint32_t kExpBits = 0x7C00u;
constexpr uint32_t kNaN2 = 0x7E007E00u;
#endif
constexpr uint32_t kNegInfBits = 0x8000u | kExpBits;  // -inf: the value of a missing entry

// Descending key: smaller key ranks first.  Any NaN -> 0xFFFF (last); +-0 -> 0x7FFF;
// otherwise key = bits ^ (sign ? 0x0000 : 0x7FFF), which is ~encode_half_asc.
__host__ __device__ __forceinline__ uint32_t desc_key(uint32_t bits) {
  bits &= 0xFFFFu;
  if ((bits & 0x7FFFu) > kExpBits) return 0xFFFFu;
  if ((bits & 0x7FFFu) == 0) return 0x7FFFu;
  return (bits & 0x8000u) ? bits : (bits ^ 0x7FFFu);
}

__device__ __forceinline__ h2t u32_as_h2(uint32_t w) {
  h2t h;
  *reinterpret_cast<uint32_t*>(&h) = w;
  return h;
}

__device__ __forceinline__ uint32_t h2_as_u32(h2t h) { return *reinterpret_cast<uint32_t*>(&h); }

// Bit pattern of the larger of the two values packed in m (a NaN half is ignored).
__device__ __forceinline__ uint32_t top_bits(uint32_t m) {
  const uint32_t sw = (m >> 16) | (m << 16);
  return h2_as_u32(__hmax2(u32_as_h2(m), u32_as_h2(sw))) & 0xFFFFu;
}

// Bit e (e = 0..7, element order) set when element e of the vector is >= v (NaN: never).
__device__ __forceinline__ uint32_t ge_mask8(const uint4& w, h2t v2) {
  const uint32_t m0 = __hge2_mask(u32_as_h2(w.x), v2);
  const uint32_t m1 = __hge2_mask(u32_as_h2(w.y), v2);
  const uint32_t m2 = __hge2_mask(u32_as_h2(w.z), v2);
  const uint32_t m3 = __hge2_mask(u32_as_h2(w.w), v2);
  const uint32_t x = (m0 & 0x00020001u) | (m1 & 0x00080004u) | (m2 & 0x00200010u) |
                     (m3 & 0x00800040u);
  return (x | (x >> 16)) & 0xFFu;
}

// Bit e set when element e is > v (NaN: never).
__device__ __forceinline__ uint32_t gt_mask8(const uint4& w, h2t v2) {
  const uint32_t m0 = __hgt2_mask(u32_as_h2(w.x), v2);
  const uint32_t m1 = __hgt2_mask(u32_as_h2(w.y), v2);
  const uint32_t m2 = __hgt2_mask(u32_as_h2(w.z), v2);
  const uint32_t m3 = __hgt2_mask(u32_as_h2(w.w), v2);
  const uint32_t x = (m0 & 0x00020001u) | (m1 & 0x00080004u) | (m2 & 0x00200010u) |
                     (m3 & 0x00800040u);
  return (x | (x >> 16)) & 0xFFu;
}

// Replace the halves whose bit is clear in valid8 by a NaN (ignored by __hmax2).
__device__ __forceinline__ uint32_t nan_fill_word(uint32_t w, uint32_t valid2) {
  const uint32_t keep = ((valid2 & 1u) ? 0x0000FFFFu : 0u) | ((valid2 & 2u) ? 0xFFFF0000u : 0u);
  return (w & keep) | (kNaN2 & ~keep);
}

__device__ __forceinline__ uint4 nan_fill(uint4 w, uint32_t valid8) {
  w.x = nan_fill_word(w.x, valid8);
  w.y = nan_fill_word(w.y, valid8 >> 2);
  w.z = nan_fill_word(w.z, valid8 >> 4);
  w.w = nan_fill_word(w.w, valid8 >> 6);
  return w;
}
