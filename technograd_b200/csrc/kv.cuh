// kv.cuh -- the KV cache's 24-bit element format.
//
// The program's keys and values are f32. The cache keeps each as its bf16 rounding h
// (2 bytes) and a signed byte q: the distance from h to x counted in the f32 bit
// pattern, in units of 256. A round-to-nearest bf16 drops the low 16 bits of x, so
// x_bits - h_bits (both with x's sign) lies in [-32768, 32768] and
//     q = round((x_bits - (h_bits << 16)) / 256)   clamped to [-127, 127],
//     x' = float from the bits (h_bits << 16) + q * 256.
// The integer form crosses binade boundaries and the subnormal range by itself, and
// |x' - x| is at most 128 f32 units in the last place of x: within 2^-16 of x relative
// to |x|. Decoding costs three integer operations per element. Decode attention reads
// 3 bytes per element instead of 4; the prefill's tensor-core attention uses h as the
// bf16 hi operand and the exact bf16 of x' - h (at most 8 significant bits) as the lo.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace tgc {

struct KvPlane {           // [slot][kv head][position][head_dim], one per layer and K/V
	__nv_bfloat16 *h;
	signed char *q;
};
struct KvPlaneC {
	const __nv_bfloat16 *h;
	const signed char *q;
};

__device__ __forceinline__ void kv_encode(float x, uint16_t &hbits, int8_t &q)
{
	const uint16_t hb = __bfloat16_as_ushort(__float2bfloat16_rn(x));
	const int d = (int)(__float_as_uint(x) - ((uint32_t)hb << 16)); // same sign: a small signed distance
	const int qi = (d + 128) >> 8;                                   // nearest multiple of 256
	hbits = hb;
	q = (int8_t)(qi > 127 ? 127 : qi < -127 ? -127 : qi);
}

// the element from its bf16 bits placed in a word's upper half and its q byte, given as a
// word whose bits 31..24 hold q (masked, then an arithmetic shift by 16 yields q * 256)
__device__ __forceinline__ float kv_decode_hq(uint32_t hi16, uint32_t q_top)
{
	return __uint_as_float(hi16 + (uint32_t)((int32_t)(q_top & 0xFF000000u) >> 16));
}

__device__ __forceinline__ float kv_decode(uint32_t hbits, int q)
{
	return __uint_as_float((hbits << 16) + (uint32_t)(q * 256));
}

// bf16 bits of the remainder x' - h (exact: at most 8 significant bits)
__device__ __forceinline__ uint32_t kv_lo_bits(uint32_t hbits, int q)
{
	const float hf = __uint_as_float(hbits << 16);
	return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(kv_decode(hbits, q) - hf));
}

// 4 consecutive elements: hi as two words (elements 0,1 | 2,3), q as one word (byte e = element e)
__device__ __forceinline__ float4 kv_decode4(uint2 h, uint32_t q)
{
	return make_float4(kv_decode_hq(h.x << 16, q << 24), kv_decode_hq(h.x & 0xFFFF0000u, q << 16),
			   kv_decode_hq(h.y << 16, q << 8), kv_decode_hq(h.y & 0xFFFF0000u, q));
}

__device__ __forceinline__ void kv_encode4(float4 x, uint2 &h, uint32_t &q)
{
	uint16_t a, b, c, d;
	int8_t qa, qb, qc, qd;
	kv_encode(x.x, a, qa), kv_encode(x.y, b, qb), kv_encode(x.z, c, qc), kv_encode(x.w, d, qd);
	h = make_uint2((uint32_t)a | ((uint32_t)b << 16), (uint32_t)c | ((uint32_t)d << 16));
	q = (uint32_t)(uint8_t)qa | ((uint32_t)(uint8_t)qb << 8) | ((uint32_t)(uint8_t)qc << 16) | ((uint32_t)(uint8_t)qd << 24);
}

} // namespace tgc
