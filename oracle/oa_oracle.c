/* CPU ORACLE for the OpenAttention decode path -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline / reference arm may load this
 * library, and only as the checker (or as the timed CPU restatement of the reference).  The product
 * (openattention_b200/) never calls it.
 *
 * A plain-C restatement of the reference's per-step algorithm (inference/methods_eager.py
 * Ours.decode :583-654, with the fused-kernel tie rules of inference/ours_fused.py and
 * inference/graph_runner.py) and of the per-request build (methods_eager.py Ours.build :505-555,
 * inference/ours_fastbuild.py :253-304).  Every floating-point operation that feeds an index
 * decision (QGS scores, codes, centroid distances, ErrorGate scores, water-filling) is written as
 * one fixed sequence of IEEE operations; the CUDA kernels perform the identical sequence, so
 * selected / expanded index sets, quotas, codes and cluster assignments must agree bit for bit.
 * Compile with -ffp-contract=off (no FMA contraction other than the explicit fmaf calls).
 *
 * Transcendentals (ln, exp, erf) are this file's own double-precision series (not libm), rounded
 * to fp32 once, so the GPU side can reproduce them exactly:
 *   ln(x)  = e*ln2 + 2*atanh(s), s = (m-1)/(m+1), m in [sqrt(1/2), sqrt(2)), 13-term odd series
 *   exp(x) = 2^k * exp(r), r = x - k*ln2 (Cody-Waite split), 17-term Taylor series
 *   erf(x) = 2/sqrt(pi) * exp(-x^2) * sum_n (2x^2)^n x / (1*3*...*(2n+1))   (all-positive series,
 *            Abramowitz & Stegun 7.1.6), 1 for x >= 6.
 * Series coefficients multiply by exact reciprocal tables (1/(2n+1), 1/i as hex literals) instead of
 * dividing, so each term costs multiplications only.
 *
 * QGS scores are exact: the int8 codes times a fixed-point image of zq summed in integers (see
 * oro_zq_fixed), so any summation order -- the GPU uses int8 tensor-core MMAs -- gives the same value.
 *
 * Layouts (contiguous): row r = b*32 + h, kv row = b*8 + h/4, D = 128.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define D 128
#define HQ 32
#define HKV 8
#define G 4
#define RQ 32
#define RC 16

/* ------------------------------------------------------------------ bf16 helpers */
static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float bfr(float f) { return bf2f(f2bf(f)); }

/* ------------------------------------------------------------------ own transcendental functions */
static const double LN2_D = 0.69314718055994530942;
static const double LN2_HI = 6.93147180369123816490e-01; /* high part, trailing zeros */
static const double LN2_LO = 1.90821492927058770002e-10;
static const double LOG2E_D = 1.44269504088896338700;

/* exact reciprocal tables (hex literals): 1/(2n+1), n = 0..400, and 1/i, i = 1..17 */
static const double INV_ODD[401] = {
    0x1.0000000000000p+0, 0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3,
    0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4, 0x1.1111111111111p-4,
    0x1.e1e1e1e1e1e1ep-5, 0x1.af286bca1af28p-5, 0x1.8618618618618p-5, 0x1.642c8590b2164p-5,
    0x1.47ae147ae147bp-5, 0x1.2f684bda12f68p-5, 0x1.1a7b9611a7b96p-5, 0x1.0842108421084p-5,
    0x1.f07c1f07c1f08p-6, 0x1.d41d41d41d41dp-6, 0x1.bacf914c1bad0p-6, 0x1.a41a41a41a41ap-6,
    0x1.8f9c18f9c18fap-6, 0x1.7d05f417d05f4p-6, 0x1.6c16c16c16c17p-6, 0x1.5c9882b931057p-6,
    0x1.4e5e0a72f0539p-6, 0x1.4141414141414p-6, 0x1.3521cfb2b78c1p-6, 0x1.29e4129e4129ep-6,
    0x1.1f7047dc11f70p-6, 0x1.15b1e5f75270dp-6, 0x1.0c9714fbcda3bp-6, 0x1.0410410410410p-6,
    0x1.f81f81f81f820p-7, 0x1.e9131abf0b767p-7, 0x1.dae6076b981dbp-7, 0x1.cd85689039b0bp-7,
    0x1.c0e070381c0e0p-7, 0x1.b4e81b4e81b4fp-7, 0x1.a98ef606a63bep-7, 0x1.9ec8e951033d9p-7,
    0x1.948b0fcd6e9e0p-7, 0x1.8acb90f6bf3aap-7, 0x1.8181818181818p-7, 0x1.78a4c8178a4c8p-7,
    0x1.702e05c0b8170p-7, 0x1.6816816816817p-7, 0x1.6058160581606p-7, 0x1.58ed2308158edp-7,
    0x1.51d07eae2f815p-7, 0x1.4afd6a052bf5bp-7, 0x1.446f86562d9fbp-7, 0x1.3e22cbce4a902p-7,
    0x1.3813813813814p-7, 0x1.323e34a2b10bfp-7, 0x1.2c9fb4d812ca0p-7, 0x1.27350b8812735p-7,
    0x1.21fb78121fb78p-7, 0x1.1cf06ada2811dp-7, 0x1.1811811811812p-7, 0x1.135c81135c811p-7,
    0x1.0ecf56be69c90p-7, 0x1.0a6810a6810a7p-7, 0x1.0624dd2f1a9fcp-7, 0x1.0204081020408p-7,
    0x1.fc07f01fc07f0p-8, 0x1.f44659e4a4271p-8, 0x1.ecc07b301ecc0p-8, 0x1.e573ac901e574p-8,
    0x1.de5d6e3f8868ap-8, 0x1.d77b654b82c34p-8, 0x1.d0cb58f6ec074p-8, 0x1.ca4b3055ee191p-8,
    0x1.c3f8f01c3f8f0p-8, 0x1.bdd2b899406f7p-8, 0x1.b7d6c3dda338bp-8, 0x1.b2036406c80d9p-8,
    0x1.ac5701ac5701bp-8, 0x1.a6d01a6d01a6dp-8, 0x1.a16d3f97a4b02p-8, 0x1.9c2d14ee4a102p-8,
    0x1.970e4f80cb872p-8, 0x1.920fb49d0e229p-8, 0x1.8d3018d3018d3p-8, 0x1.886e5f0abb04ap-8,
    0x1.83c977ab2beddp-8, 0x1.7f405fd017f40p-8, 0x1.7ad2208e0ecc3p-8, 0x1.767dce434a9b1p-8,
    0x1.724287f46debcp-8, 0x1.6e1f76b4337c7p-8, 0x1.6a13cd1537290p-8, 0x1.661ec6a5122f9p-8,
    0x1.623fa77016240p-8, 0x1.5e75bb8d015e7p-8, 0x1.5ac056b015ac0p-8, 0x1.571ed3c506b3ap-8,
    0x1.5390948f40febp-8, 0x1.5015015015015p-8, 0x1.4cab88725af6ep-8, 0x1.49539e3b2d067p-8,
    0x1.460cbc7f5cf9ap-8, 0x1.42d6625d51f87p-8, 0x1.3fb013fb013fbp-8, 0x1.3c995a47babe7p-8,
    0x1.3991c2c187f63p-8, 0x1.3698df3de0748p-8, 0x1.33ae45b57bcb2p-8, 0x1.30d190130d190p-8,
    0x1.2e025c04b8097p-8, 0x1.2b404ad012b40p-8, 0x1.288b01288b013p-8, 0x1.25e22708092f1p-8,
    0x1.23456789abcdfp-8, 0x1.20b470c67c0d9p-8, 0x1.1e2ef3b3fb874p-8, 0x1.1bb4a4046ed29p-8,
    0x1.19453808ca29cp-8, 0x1.16e0689427379p-8, 0x1.1485f0e0acd3bp-8, 0x1.12358e75d3033p-8,
    0x1.0fef010fef011p-8, 0x1.0db20a88f4696p-8, 0x1.0b7e6ec259dc8p-8, 0x1.0953f39010954p-8,
    0x1.073260a47f7c6p-8, 0x1.05197f7d73404p-8, 0x1.03091b51f5e1ap-8, 0x1.0101010101010p-8,
    0x1.fe01fe01fe020p-9, 0x1.fa11caa01fa12p-9, 0x1.f6310aca0dbb5p-9, 0x1.f25f644230ab5p-9,
    0x1.ee9c7f8458e02p-9, 0x1.eae807aba01ebp-9, 0x1.e741aa59750e4p-9, 0x1.e3a9179dc1a73p-9,
    0x1.e01e01e01e01ep-9, 0x1.dca01dca01dcap-9, 0x1.d92f2231e7f8ap-9, 0x1.d5cac807572b2p-9,
    0x1.d272ca3fc5b1ap-9, 0x1.cf26e5c44bfc6p-9, 0x1.cbe6d9601cbe7p-9, 0x1.c8b265afb8a42p-9,
    0x1.c5894d10d4986p-9, 0x1.c26b5392ea01cp-9, 0x1.bf583ee868d8bp-9, 0x1.bc4fd65883e7bp-9,
    0x1.b951e2b18ff23p-9, 0x1.b65e2e3beee05p-9, 0x1.b37484ad806cep-9, 0x1.b094b31d922a4p-9,
    0x1.adbe87f94905ep-9, 0x1.aaf1d2f87ebfdp-9, 0x1.a82e65130e159p-9, 0x1.a574107688a4ap-9,
    0x1.a2c2a87c51ca0p-9, 0x1.a01a01a01a01ap-9, 0x1.9d79f176b682dp-9, 0x1.9ae24ea5510dap-9,
    0x1.9852f0d8ec0ffp-9, 0x1.95cbb0be377aep-9, 0x1.934c67f9b2ce6p-9, 0x1.90d4f120190d5p-9,
    0x1.8e6527af1373fp-9, 0x1.8bfce8062ff3ap-9, 0x1.899c0f601899cp-9, 0x1.87427bcc092b9p-9,
    0x1.84f00c2780614p-9, 0x1.82a4a0182a4a0p-9, 0x1.8060180601806p-9, 0x1.7e225515a4f1dp-9,
    0x1.7beb3922e017cp-9, 0x1.79baa6bb6398bp-9, 0x1.77908119ac60dp-9, 0x1.756cac201756dp-9,
    0x1.734f0c541fe8dp-9, 0x1.713786d9c7c09p-9, 0x1.6f26016f26017p-9, 0x1.6d1a62681c861p-9,
    0x1.6b1490aa31a3dp-9, 0x1.691473a88d0c0p-9, 0x1.6719f3601671ap-9, 0x1.6524f853b4aa3p-9,
    0x1.63356b88ac0dep-9, 0x1.614b36831ae94p-9, 0x1.5f66434292dfcp-9, 0x1.5d867c3ece2a5p-9,
    0x1.5babcc647fa91p-9, 0x1.59d61f123ccaap-9, 0x1.5805601580560p-9, 0x1.56397ba7c52e2p-9,
    0x1.54725e6bb82fep-9, 0x1.52aff56a8054bp-9, 0x1.50f22e111c4c5p-9, 0x1.4f38f62dd4c9bp-9,
    0x1.4d843bedc2c4cp-9, 0x1.4bd3edda68fe1p-9, 0x1.4a27fad76014ap-9, 0x1.4880522014880p-9,
    0x1.46dce34596066p-9, 0x1.453d9e2c776cap-9, 0x1.43a2730abee4dp-9, 0x1.420b5265e5951p-9,
    0x1.40782d10e6566p-9, 0x1.3ee8f42a5af07p-9, 0x1.3d5d991aa75c6p-9, 0x1.3bd60d9232955p-9,
    0x1.3a524387ac822p-9, 0x1.38d22d366088ep-9, 0x1.3755bd1c945eep-9, 0x1.35dce5f9f2af8p-9,
    0x1.34679ace01346p-9, 0x1.32f5ced6a1dfap-9, 0x1.3187758e9ebb6p-9, 0x1.301c82ac40260p-9,
    0x1.2eb4ea1fed14bp-9, 0x1.2d50a012d50a0p-9, 0x1.2bef98e5a3711p-9, 0x1.2a91c92f3c105p-9,
    0x1.293725bb804a5p-9, 0x1.27dfa38a1ce4dp-9, 0x1.268b37cd60127p-9, 0x1.2539d7e9177b2p-9,
    0x1.23eb79717605bp-9, 0x1.22a0122a0122ap-9, 0x1.21579804855e6p-9, 0x1.2012012012012p-9,
    0x1.1ecf43c7fb84cp-9, 0x1.1d8f5672e4abdp-9, 0x1.1c522fc1ce059p-9, 0x1.1b17c67f2bae3p-9,
    0x1.19e0119e0119ep-9, 0x1.18ab083902bdbp-9, 0x1.1778a191bd684p-9, 0x1.1648d50fc3201p-9,
    0x1.151b9a3fdd5c9p-9, 0x1.13f0e8d344724p-9, 0x1.12c8b89edc0acp-9, 0x1.11a3019a74826p-9,
    0x1.107fbbe011080p-9, 0x1.0f5edfab325a2p-9, 0x1.0e40655826011p-9, 0x1.0d24456359e3ap-9,
    0x1.0c0a7868b4171p-9, 0x1.0af2f722eecb5p-9, 0x1.09ddba6af8360p-9, 0x1.08cabb37565e2p-9,
    0x1.07b9f29b8eae2p-9, 0x1.06ab59c7912fbp-9, 0x1.059eea0727586p-9, 0x1.04949cc1664c5p-9,
    0x1.038c6b78247fcp-9, 0x1.02864fc7729e9p-9, 0x1.0182436517a37p-9, 0x1.0080402010080p-9,
    0x1.ff007fc01ff00p-10, 0x1.fd04794a10e6ap-10, 0x1.fb0c610d5e939p-10, 0x1.f9182b6813bafp-10,
    0x1.f727cce5f530ap-10, 0x1.f53b3a3fa204ep-10, 0x1.f3526859b8cecp-10, 0x1.f16d4c4401f17p-10,
    0x1.ef8bdb389ebadp-10, 0x1.edae0a9b3d3a5p-10, 0x1.ebd3cff850b0cp-10, 0x1.e9fd21044e799p-10,
    0x1.e829f39aef509p-10, 0x1.e65a3dbe74d6bp-10, 0x1.e48df596f3394p-10, 0x1.e2c511719ee16p-10,
    0x1.e0ff87c01e100p-10, 0x1.df3d4f17de4dbp-10, 0x1.dd7e5e316d94cp-10, 0x1.dbc2abe7d71d4p-10,
    0x1.da0a2f3803b41p-10, 0x1.d854df401d855p-10, 0x1.d6a2b33ef7448p-10, 0x1.d4f3a293769cap-10,
    0x1.d347a4bc01d34p-10, 0x1.d19eb155f08a4p-10, 0x1.cff8c01cff8c0p-10, 0x1.ce55c8eac7900p-10,
    0x1.ccb5c3b636e3ap-10, 0x1.cb18a8930de60p-10, 0x1.c97e6fb15e44dp-10, 0x1.c7e7115d0ce95p-10,
    0x1.c65285fd56843p-10, 0x1.c4c0c61456a8ep-10, 0x1.c331ca3e91679p-10, 0x1.c1a58b327f576p-10,
    0x1.c01c01c01c01cp-10, 0x1.be9526d0769fap-10, 0x1.bd10f365451b6p-10, 0x1.bb8f609879493p-10,
    0x1.ba10679bd8488p-10, 0x1.b89401b89401cp-10, 0x1.b71a284ee6b34p-10, 0x1.b5a2d4d5b081fp-10,
    0x1.b42e00da17007p-10, 0x1.b2bba5ff26a23p-10, 0x1.b14bbdfd760e6p-10, 0x1.afde42a2cb482p-10,
    0x1.ae732dd1c2a09p-10, 0x1.ad0a798177693p-10, 0x1.aba41fbd2e5b1p-10, 0x1.aa401aa401aa4p-10,
    0x1.a8de64688ebabp-10, 0x1.a77ef750a56dap-10, 0x1.a621cdb4f8fdfp-10, 0x1.a4c6e200d2637p-10,
    0x1.a36e2eb1c432dp-10, 0x1.a217ae575ff2fp-10, 0x1.a0c35b92ecdf1p-10, 0x1.9f713117200d0p-10,
    0x1.9e2129a7d5f0ap-10, 0x1.9cd34019cd340p-10, 0x1.9b876f5262dd1p-10, 0x1.9a3db2474fb98p-10,
    0x1.98f603fe670a0p-10, 0x1.97b05f8d56652p-10, 0x1.966cc01966cc0p-10, 0x1.952b20d73ee97p-10,
    0x1.93eb7d0aa6759p-10, 0x1.92add0064ab74p-10, 0x1.9172152b841ddp-10, 0x1.903847ea1cec1p-10,
    0x1.8f0063c018f00p-10, 0x1.8dca64397e408p-10, 0x1.8c9644f01efbcp-10, 0x1.8b64018b64019p-10,
    0x1.8a3395c018a34p-10, 0x1.8904fd503744bp-10, 0x1.87d8340ab6e97p-10, 0x1.86ad35cb59a84p-10,
    0x1.8583fe7a7c018p-10, 0x1.845c8a0ce5129p-10, 0x1.8336d48397a24p-10, 0x1.8212d9eba4018p-10,
    0x1.80f0965dfabcbp-10, 0x1.7fd005ff40180p-10, 0x1.7eb124ffa053bp-10, 0x1.7d93ef9aa4b46p-10,
    0x1.7c7862170949fp-10, 0x1.7b5e78c693733p-10, 0x1.7a463005e918cp-10, 0x1.792f843c689c3p-10,
    0x1.781a71dc01782p-10, 0x1.7706f5610d8d0p-10, 0x1.75f50b522b17cp-10, 0x1.74e4b040174e5p-10,
    0x1.73d5e0c5899f7p-10, 0x1.72c899870f91fp-10, 0x1.71bcd732e940ap-10, 0x1.70b29680e66fap-10,
    0x1.6fa9d43244380p-10, 0x1.6ea28d118b474p-10, 0x1.6d9cbdf26eaefp-10, 0x1.6c9863b1ab429p-10,
    0x1.6b957b34e7803p-10, 0x1.6a94016a94017p-10, 0x1.6993f349cc726p-10, 0x1.68954dd2390bap-10,
    0x1.67980e0bf08c7p-10, 0x1.669c31075ab40p-10, 0x1.65a1b3dd13357p-10, 0x1.64a893adcd25fp-10,
    0x1.63b0cda236e1cp-10, 0x1.62ba5eeade65ep-10, 0x1.61c544c0161c5p-10, 0x1.60d17c61da198p-10,
    0x1.5fdf0317b5c6fp-10, 0x1.5eedd630a9fb3p-10, 0x1.5dfdf303137b6p-10, 0x1.5d0f56ec91e57p-10,
    0x1.5c21ff51ef005p-10, 0x1.5b35e99f06714p-10, 0x1.5a4b1346add2bp-10, 0x1.596179c29d2cep-10,
    0x1.58791a9357ccep-10, 0x1.5791f34015792p-10, 0x1.56ac0156ac015p-10, 0x1.55c7426b79286p-10,
    0x1.54e3b4194ce66p-10, 0x1.5401540154015p-10, 0x1.53201fcb02fb1p-10, 0x1.5240152401524p-10,
    0x1.516131c015161p-10, 0x1.508373590ec9cp-10, 0x1.4fa6d7aeb597cp-10, 0x1.4ecb5c86b3d24p-10,
    0x1.4df0ffac83c01p-10, 0x1.4d17bef15cb4ep-10, 0x1.4c3f982c20723p-10, 0x1.4b68893948d1cp-10,
    0x1.4a928ffad5b5cp-10, 0x1.49bdaa583b401p-10, 0x1.48e9d63e504d1p-10, 0x1.4817119f3d325p-10,
    0x1.47455a726abf2p-10,
};
static const double INV_INT[18] = {
    0x0p+0, 0x1.0000000000000p+0, 0x1.0000000000000p-1, 0x1.5555555555555p-2,
    0x1.0000000000000p-2, 0x1.999999999999ap-3, 0x1.5555555555555p-3, 0x1.2492492492492p-3,
    0x1.0000000000000p-3, 0x1.c71c71c71c71cp-4, 0x1.999999999999ap-4, 0x1.745d1745d1746p-4,
    0x1.5555555555555p-4, 0x1.3b13b13b13b14p-4, 0x1.2492492492492p-4, 0x1.1111111111111p-4,
    0x1.0000000000000p-4, 0x1.e1e1e1e1e1e1ep-5,
};

static double pow2i(int k) { /* exact 2^k for -1022 <= k <= 1023 */
  uint64_t bits = (uint64_t)(k + 1023) << 52;
  double d;
  memcpy(&d, &bits, 8);
  return d;
}

double oro_ln_d(double x) { /* x > 0, normal */
  uint64_t bits;
  memcpy(&bits, &x, 8);
  int e = (int)((bits >> 52) & 0x7ff) - 1022;
  bits = (bits & 0x000fffffffffffffull) | 0x3fe0000000000000ull; /* m in [0.5, 1) */
  double m;
  memcpy(&m, &bits, 8);
  if (m < 0.70710678118654752440) {
    m = m * 2.0;
    e = e - 1;
  }
  double s = (m - 1.0) / (m + 1.0);
  double s2 = s * s;
  double term = s, sum = s;
  for (int k = 1; k <= 13; ++k) {
    term = term * s2;
    sum = sum + term * INV_ODD[k];
  }
  double a = 2.0 * sum;
  double b = (double)e * LN2_D;
  return a + b;
}

double oro_exp_d(double x) {
  if (x < -745.0) return 0.0;
  if (x > 709.0) return INFINITY;
  double k = nearbyint(x * LOG2E_D);
  double t1 = k * LN2_HI;
  double t2 = k * LN2_LO;
  double r = (x - t1) - t2;
  double p = 1.0, term = 1.0;
  for (int i = 1; i <= 17; ++i) {
    term = term * r;
    term = term * INV_INT[i];
    p = p + term;
  }
  int ki = (int)k;
  if (ki < -1022) return 0.0;
  return p * pow2i(ki);
}

double oro_erf_d(double x) { /* x >= 0 */
  if (x >= 6.0) return 1.0;
  double x2 = x * x;
  double tx2 = 2.0 * x2;
  double term = x, sum = x;
  for (int n = 1; n < 400; ++n) {
    term = term * tx2;
    term = term * INV_ODD[n];
    sum = sum + term;
    if (term < sum * 1e-17) break;
  }
  double c = 1.1283791670955126 * oro_exp_d(-x2);
  return c * sum;
}

float oro_logf(float x) { return (float)oro_ln_d((double)x); }
float oro_expf(float x) {
  if (x == -INFINITY) return 0.0f;
  return (float)oro_exp_d((double)x);
}
/* From x = 4 on the series rounds to 1 in fp32 (erf(x) > 1 - 1.6e-8, the series is accurate to about
 * 1e-14, and the fp32 midpoint below 1 is 1 - 3e-8): both implementations skip it there. */
float oro_erff(float x) { return x >= 4.0f ? 1.0f : (float)oro_erf_d((double)x); }

/* ------------------------------------------------------------------ decode: index update */
/* New token at position pos of every request: QGS code (per KV head), nearest QGC centroid (per
 * query head, ties -> lower id), n_b += 1, Sk += k, Sk2 += k*k, Sv += v, generated-token list append.
 * Restates ours_graph._k_index_update_d2 (inference/ours_graph.py:43-90) / methods_eager.py:586-601. */
void oro_index_update(int B, int Lmax, int C, int pos, const uint16_t* K, const uint16_t* V, int8_t* codes,
                      const float* U, const float* scale, const uint16_t* W, const float* colmean,
                      const float* cent, int32_t* asg, float* nb, float* Sk, float* Sk2, float* Sv,
                      int32_t* reclist, int32_t* reccnt, int rmax) {
  for (int kv = 0; kv < B * HKV; ++kv) {
    const uint16_t* kr = K + ((int64_t)kv * Lmax + pos) * D;
    const uint16_t* vr = V + ((int64_t)kv * Lmax + pos) * D;
    float kf[D], vf[D];
    for (int d = 0; d < D; ++d) {
      kf[d] = bf2f(kr[d]);
      vf[d] = bf2f(vr[d]);
    }
    const float* Uk = U + (int64_t)kv * D * RQ;
    for (int j = 0; j < RQ; ++j) {
      float acc = 0.0f;
      for (int d = 0; d < D; ++d) acc = fmaf(kf[d], Uk[d * RQ + j], acc);
      float c = rintf(acc / scale[kv * RQ + j]);
      c = fminf(fmaxf(c, -127.0f), 127.0f);
      codes[((int64_t)kv * Lmax + pos) * RQ + j] = (int8_t)c;
    }
    for (int g = 0; g < G; ++g) {
      const int r = kv * G + g;
      const uint16_t* Wr = W + (int64_t)r * D * RC;
      float zp[RC];
      for (int c = 0; c < RC; ++c) {
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc = fmaf(kf[d], bf2f(Wr[d * RC + c]), acc);
        zp[c] = bfr(acc) - colmean[r * RC + c];
      }
      const float* ce = cent + (int64_t)r * C * RC;
      int best = 0;
      float bestv = -INFINITY;
      for (int i = 0; i < C; ++i) {
        float dot = 0.0f, nrm = 0.0f;
        for (int c = 0; c < RC; ++c) {
          dot = fmaf(zp[c], ce[i * RC + c], dot);
          nrm = fmaf(ce[i * RC + c], ce[i * RC + c], nrm);
        }
        float dist = dot - 0.5f * nrm;
        if (dist > bestv) {
          bestv = dist;
          best = i;
        }
      }
      asg[(int64_t)r * Lmax + pos] = best;
      nb[r * C + best] += 1.0f;
      float* sk = Sk + ((int64_t)r * C + best) * D;
      float* sk2 = Sk2 + ((int64_t)r * C + best) * D;
      float* sv = Sv + ((int64_t)r * C + best) * D;
      for (int d = 0; d < D; ++d) {
        sk[d] = sk[d] + kf[d];
        float kk = kf[d] * kf[d];
        sk2[d] = sk2[d] + kk;
        sv[d] = sv[d] + vf[d];
      }
      if (reclist) {
        int cnt = reccnt[r * C + best];
        if (cnt < rmax) reclist[((int64_t)r * C + best) * rmax + cnt] = pos;
        reccnt[r * C + best] = cnt + 1;
      }
    }
  }
}

/* zq[r, j] = bf16((q_r . U[:, j]) * scale_j), U of the row's KV head (methods_eager.py:603). */
void oro_zq(int B, const uint16_t* q, const float* U, const float* scale, uint16_t* zq) {
  for (int r = 0; r < B * HQ; ++r) {
    const int kv = r / G;
    float qf[D];
    for (int d = 0; d < D; ++d) qf[d] = bf2f(q[(int64_t)r * D + d]);
    for (int j = 0; j < RQ; ++j) {
      float acc = 0.0f;
      for (int d = 0; d < D; ++d) acc = fmaf(qf[d], U[((int64_t)kv * D + d) * RQ + j], acc);
      float z = acc * scale[kv * RQ + j];
      zq[r * RQ + j] = f2bf(z);
    }
  }
}

/* Exact fixed-point image of one query head's zq (32 bf16 values): Z_j = trunc(z_j * 2^S) with
 * S = 29 - e_max (e_max = binary exponent of max |z_j|), so |Z_j| < 2^30; z_j below 2^(e_max - 23)
 * lose their fractional bits.  Returns S; all-zero (or below 2^-100) heads give S = 0, Z = 0. */
static float pow2f_exact(int k) { /* 2^k as float, -126 <= k <= 127 */
  uint32_t b = (uint32_t)(k + 127) << 23;
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static float scale_pow2(float x, int k) { /* x * 2^k by exact power-of-two steps */
  while (k > 100) { x = x * pow2f_exact(100); k -= 100; }
  while (k < -100) { x = x * pow2f_exact(-100); k += 100; }
  return x * pow2f_exact(k);
}
int oro_zq_fixed(const uint16_t* zq, int32_t* Z) {
  float amax = 0.0f;
  for (int j = 0; j < RQ; ++j) {
    float a = fabsf(bf2f(zq[j]));
    if (a > amax) amax = a;
  }
  uint32_t ab;
  memcpy(&ab, &amax, 4);
  const int e_max = (int)((ab >> 23) & 0xff) - 127;
  if (amax == 0.0f || e_max < -100) {
    for (int j = 0; j < RQ; ++j) Z[j] = 0;
    return 0;
  }
  const int S = 29 - e_max;
  for (int j = 0; j < RQ; ++j) Z[j] = (int32_t)scale_pow2(bf2f(zq[j]), S); /* C cast truncates */
  return S;
}

/* QGS scores s[r, t] = bf16( fp32( sum_j code[t, j] * Z[r, j] ) * 2^-S_r ): the exact integer dot
 * product of the int8 codes with the fixed-point zq, rounded once to fp32 and once to bf16 (the
 * value an fp32 sum without intermediate rounding would give); -inf for t < ns and t >= n - nl.
 * Restates _k_qgs_scan_tm (inference/graph_runner.py:100-120). s: (R, sw) bf16 bits. */
void oro_scan(int B, int Lmax, int n, int ns, int nl, const int8_t* codes, const uint16_t* zq, uint16_t* s,
              int64_t sw) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < B * HQ; ++r) {
    const int kv = r / G;
    int32_t Z[RQ];
    const int S = oro_zq_fixed(zq + (int64_t)r * RQ, Z);
    const int8_t* cr = codes + (int64_t)kv * Lmax * RQ;
    uint16_t* sr = s + (int64_t)r * sw;
    for (int t = 0; t < n; ++t) {
      int64_t acc = 0;
      const int8_t* c = cr + (int64_t)t * RQ;
      for (int j = 0; j < RQ; ++j) acc += (int64_t)c[j] * (int64_t)Z[j];
      const float f = scale_pow2((float)acc, -S);
      uint16_t v = f2bf(f);
      if (t < ns || t >= n - nl) v = 0xff80; /* -inf */
      sr[t] = v;
    }
  }
}

/* orderable 16-bit key of a bf16 score: larger score -> larger key */
static inline uint32_t ukey16(uint16_t b) { return (b & 0x8000u) ? (uint32_t)(~b & 0xffffu) : (uint32_t)(b | 0x8000u); }

/* Row top-k by (score desc, position asc); sel = [0..ns-1, n-nl..n-1, top (in rank order)]; the
 * selected scores are then set to -inf.  Restates _k_select (inference/graph_runner.py:123-159). */
void oro_select(int R, int n, int ns, int nl, int k_top, uint16_t* s, int64_t sw, int32_t* sel) {
  const int NS = ns + nl + k_top;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < R; ++r) {
    uint16_t* sr = s + (int64_t)r * sw;
    int32_t* o = sel + (int64_t)r * NS;
    for (int i = 0; i < ns; ++i) o[i] = i;
    for (int i = 0; i < nl; ++i) o[ns + i] = n - nl + i;
    /* insertion into a sorted top list (k_top is small) */
    int32_t* top = o + ns + nl;
    uint32_t tk[4096];
    if (k_top > 4096) k_top = 4096;
    int cnt = 0;
    for (int t = 0; t < n; ++t) {
      uint32_t key = ukey16(sr[t]);
      if (cnt == k_top && key <= tk[cnt - 1]) continue; /* ties keep the lower position */
      int p = cnt < k_top ? cnt : k_top - 1;
      while (p > 0 && tk[p - 1] < key) {
        tk[p] = tk[p - 1];
        top[p] = top[p - 1];
        --p;
      }
      tk[p] = key;
      top[p] = t;
      if (cnt < k_top) ++cnt;
    }
    for (int i = 0; i < k_top; ++i) sr[top[i]] = 0xff80;
  }
}

/* 128-term dot product in the order one warp computes it: lane l holds dims 4l .. 4l+3 and
 * accumulates fma(a[4l+3], b[4l+3], fma(a[4l+2], b[4l+2], fma(a[4l+1], b[4l+1], a[4l]*b[4l]))), then
 * the 32 partials are combined by an xor butterfly over offsets 16, 8, 4, 2, 1. */
float oro_dot128_tree(const float* a, const float* b) {
  float p[32], t[32];
  for (int l = 0; l < 32; ++l) {
    float v = a[4 * l] * b[4 * l];
    v = fmaf(a[4 * l + 1], b[4 * l + 1], v);
    v = fmaf(a[4 * l + 2], b[4 * l + 2], v);
    v = fmaf(a[4 * l + 3], b[4 * l + 3], v);
    p[l] = v;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    for (int l = 0; l < 32; ++l) t[l] = p[l] + p[l ^ off];
    for (int l = 0; l < 32; ++l) p[l] = t[l];
  }
  return p[0];
}

/* ErrorGate wl1 (inference/ours_fused.py:122-154, methods_eager.py:613-627).  Per row: tail sums
 * (pooled sums minus the selected tokens, in sel order), then per cluster
 *   kbar = Skt*inv, var = max(Sk2t*inv - kbar*kbar, 0), inv = 1/max(nt,1)
 *   zbar = SC * dot(q, kbar),  s2 = SC^2 * dot(q*q, var)   (oro_dot128_tree order)
 *   score = ((zbar + ln max(nt,1)) + 0.5 s2) + ln max(erf(sqrt(s2)*0.70710677), 1e-30). */
void oro_errorgate(int B, int Lmax, int C, int NS, const uint16_t* q, const uint16_t* K, const int32_t* asg,
                   const int32_t* sel, const float* Sk, const float* Sk2, const float* nb, float* score, float* nt) {
  const float SCf = 0.08838834764831845f;
  const float SC2f = 0.0078125f;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < B * HQ; ++r) {
    const int kv = r / G;
    float* skt = (float*)malloc(sizeof(float) * C * D);
    float* sk2t = (float*)malloc(sizeof(float) * C * D);
    memcpy(skt, Sk + (int64_t)r * C * D, sizeof(float) * C * D);
    memcpy(sk2t, Sk2 + (int64_t)r * C * D, sizeof(float) * C * D);
    float* ntr = nt + (int64_t)r * C;
    for (int c = 0; c < C; ++c) ntr[c] = nb[(int64_t)r * C + c];
    for (int j = 0; j < NS; ++j) {
      const int t = sel[(int64_t)r * NS + j];
      const int c = asg[(int64_t)r * Lmax + t];
      const uint16_t* kr = K + ((int64_t)kv * Lmax + t) * D;
      for (int d = 0; d < D; ++d) {
        float kf = bf2f(kr[d]);
        skt[c * D + d] = skt[c * D + d] - kf;
        float kk = kf * kf;
        sk2t[c * D + d] = sk2t[c * D + d] - kk;
      }
      ntr[c] = ntr[c] - 1.0f;
    }
    float qf[D], q2[D];
    for (int d = 0; d < D; ++d) {
      qf[d] = bf2f(q[(int64_t)r * D + d]);
      q2[d] = qf[d] * qf[d];
    }
    for (int c = 0; c < C; ++c) {
      const float inv = 1.0f / fmaxf(ntr[c], 1.0f);
      float kb[D], var[D];
      for (int d = 0; d < D; ++d) {
        kb[d] = skt[c * D + d] * inv;
        float p1 = sk2t[c * D + d] * inv;
        float p2 = kb[d] * kb[d];
        var[d] = fmaxf(p1 - p2, 0.0f);
      }
      float zd = oro_dot128_tree(qf, kb);
      float sd = oro_dot128_tree(q2, var);
      float zbar = SCf * zd;
      float s2 = SC2f * sd;
      float lg = oro_logf(fmaxf(ntr[c], 1.0f));
      float er = oro_erff(sqrtf(s2) * 0.70710677f);
      float le = oro_logf(fmaxf(er, 1e-30f));
      float hs = 0.5f * s2;
      float sc = zbar + lg;
      sc = sc + hs;
      sc = sc + le;
      score[(int64_t)r * C + c] = sc;
    }
    free(skt);
    free(sk2t);
  }
}

/* Hierarchical water-filling (inference/ours_fused.py:158-216 = methods_eager.py Ours.hier_quota
 * :558-581).  Sorts by (ratio asc, cluster asc) and (score desc, cluster asc); suffix sums of the
 * weights accumulate in double from the end (as torch's CPU cumsum does for fp32). */
void oro_waterfill(int R, int C, float E, const float* score, const float* nt, float* quota) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < R; ++r) {
    const float* sc = score + (int64_t)r * C;
    const float* n_t = nt + (int64_t)r * C;
    float* qo = quota + (int64_t)r * C;
    float s[256], w[256], cap[256], ratio[256], qb[256];
    int o[256], o2[256];
    float smax = -INFINITY;
    int any = 0;
    for (int c = 0; c < C; ++c) {
      int live = n_t[c] > 1.0f;
      s[c] = live ? sc[c] : -INFINITY;
      if (live) any = 1;
      if (s[c] > smax) smax = s[c];
    }
    float tot = 0.0f;
    for (int c = 0; c < C; ++c) {
      int live = n_t[c] > 1.0f;
      w[c] = live ? oro_expf(s[c] - smax) : 0.0f;
      cap[c] = live ? n_t[c] : 0.0f;
      tot = tot + cap[c];
      ratio[c] = w[c] > 0.0f ? cap[c] / fmaxf(w[c], 1e-30f) : INFINITY;
    }
    (void)any;
    /* stable insertion sort by ratio asc (index order kept among equal ratios) */
    for (int c = 0; c < C; ++c) {
      int p = c;
      while (p > 0 && ratio[o[p - 1]] > ratio[c]) {
        o[p] = o[p - 1];
        --p;
      }
      o[p] = c;
    }
    float c_ex[256], w_suf[256];
    float run = 0.0f;
    for (int j = 0; j < C; ++j) {
      c_ex[j] = run;
      run = run + cap[o[j]];
    }
    double acc = 0.0;
    for (int j = C - 1; j >= 0; --j) {
      acc = acc + (double)w[o[j]];
      w_suf[j] = (float)acc;
    }
    int jj = -1;
    for (int j = 0; j < C; ++j) {
      float f;
      if (w_suf[j] > 0.0f) {
        float prod = ratio[o[j]] * w_suf[j];
        f = c_ex[j] + prod;
      } else {
        f = INFINITY;
      }
      if (f >= E) {
        jj = j;
        break;
      }
    }
    if (jj < 0) jj = 0;
    const float lam = (E - c_ex[jj]) / fmaxf(w_suf[jj], 1e-30f);
    float sumq = 0.0f;
    for (int c = 0; c < C; ++c) {
      float lw = lam * w[c];
      qb[c] = fminf(cap[c], floorf(lw));
      if (tot <= E) qb[c] = cap[c];
      sumq = sumq + qb[c];
    }
    float rem = fmaxf(fminf(tot, E) - sumq, 0.0f);
    /* leftover: score desc, cluster asc */
    for (int c = 0; c < C; ++c) {
      int p = c;
      while (p > 0 && s[o2[p - 1]] < s[c]) {
        o2[p] = o2[p - 1];
        --p;
      }
      o2[p] = c;
    }
    int given = 0;
    for (int i = 0; i < C; ++i) {
      const int c = o2[i];
      float add = 0.0f;
      if (qb[c] < cap[c]) {
        if ((float)given < rem) add = 1.0f;
        ++given;
      }
      qo[c] = qb[c] + add;
    }
  }
}

/* Within-cluster top-q (inference/ours_graph.py:93-166, ours_fused.py:220-363): for each cluster c
 * with quota q > 0, its members (prefix tokens t < n0 and generated tokens n0 <= t < n with
 * asg == c) ranked by (score desc, position asc); the first q are written to
 * exp[r, base_c : base_c + q] in ascending position, base_c = sum of the quotas of clusters < c.
 * Unused slots are -1. */
void oro_topq(int R, int Lmax, int C, int E, int n, const uint16_t* s, int64_t sw, const int32_t* asg,
              const float* quota, int32_t* exp_idx) {
#pragma omp parallel for schedule(dynamic, 4)
  for (int r = 0; r < R; ++r) {
    const uint16_t* sr = s + (int64_t)r * sw;
    const int32_t* ar = asg + (int64_t)r * Lmax;
    const float* qr = quota + (int64_t)r * C;
    int32_t* er = exp_idx + (int64_t)r * E;
    for (int i = 0; i < E; ++i) er[i] = -1;
    /* bucket the row's tokens by cluster, each bucket in ascending position */
    int32_t* start = (int32_t*)calloc((size_t)C + 1, sizeof(int32_t));
    int32_t* fill = (int32_t*)calloc((size_t)C, sizeof(int32_t));
    int32_t* tok = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    for (int t = 0; t < n; ++t) start[ar[t] + 1]++;
    for (int c = 0; c < C; ++c) start[c + 1] += start[c];
    for (int t = 0; t < n; ++t) {
      const int c = ar[t];
      tok[start[c] + fill[c]++] = t;
    }
    int base = 0;
    for (int c = 0; c < C; ++c) {
      const int q = (int)qr[c];
      if (q <= 0) continue;
      const int32_t* mt = tok + start[c];
      const int m = start[c + 1] - start[c];
      /* two 8-bit radix passes find the threshold key T (the q-th largest) */
      int hist[256];
      memset(hist, 0, sizeof(hist));
      for (int i = 0; i < m; ++i) hist[ukey16(sr[mt[i]]) >> 8]++;
      int above = 0, hi = 0;
      for (int b = 255; b >= 0; --b) {
        if (above + hist[b] >= q) {
          hi = b;
          break;
        }
        above += hist[b];
      }
      memset(hist, 0, sizeof(hist));
      for (int i = 0; i < m; ++i) {
        const uint32_t k = ukey16(sr[mt[i]]);
        if ((int)(k >> 8) == hi) hist[k & 255]++;
      }
      int lo = 0;
      for (int b = 255; b >= 0; --b) {
        if (above + hist[b] >= q) {
          lo = b;
          break;
        }
        above += hist[b];
      }
      const uint32_t T = ((uint32_t)hi << 8) | (uint32_t)lo;
      int need = q - above, w = 0;
      for (int i = 0; i < m && w < q; ++i) {
        const uint32_t k = ukey16(sr[mt[i]]);
        if (k > T || (k == T && need > 0)) {
          if (k == T) --need;
          if (base + w < E) er[base + w] = mt[i];
          ++w;
        }
      }
      base += q;
    }
    free(start);
    free(fill);
    free(tok);
  }
}

/* Residual proxies (inference/ours_fused.py:367-407, methods_eager.py:641-652): pooled sums minus
 * every token read (sel in order, then exp slots in order; -1 slots skipped), n' = nt - quota,
 * kbar' = bf16(Skr/max(n',1)), vbar' = bf16(Svr/max(n',1)), log n' = ln max(n',1) if n' > 0.5 else -inf. */
void oro_residual(int B, int Lmax, int C, int NS, int E, const uint16_t* K, const uint16_t* V, const int32_t* asg,
                  const int32_t* sel, const int32_t* exp_idx, const float* Sk, const float* Sv, const float* nt,
                  const float* quota, uint16_t* kbar, uint16_t* vbar, float* logn) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < B * HQ; ++r) {
    const int kv = r / G;
    float* skr = (float*)malloc(sizeof(float) * C * D);
    float* svr = (float*)malloc(sizeof(float) * C * D);
    memcpy(skr, Sk + (int64_t)r * C * D, sizeof(float) * C * D);
    memcpy(svr, Sv + (int64_t)r * C * D, sizeof(float) * C * D);
    for (int j = 0; j < NS + E; ++j) {
      const int t = j < NS ? sel[(int64_t)r * NS + j] : exp_idx[(int64_t)r * E + (j - NS)];
      if (t < 0) continue;
      const int c = asg[(int64_t)r * Lmax + t];
      const uint16_t* kr = K + ((int64_t)kv * Lmax + t) * D;
      const uint16_t* vr = V + ((int64_t)kv * Lmax + t) * D;
      for (int d = 0; d < D; ++d) {
        skr[c * D + d] = skr[c * D + d] - bf2f(kr[d]);
        svr[c * D + d] = svr[c * D + d] - bf2f(vr[d]);
      }
    }
    for (int c = 0; c < C; ++c) {
      const float nr = nt[(int64_t)r * C + c] - quota[(int64_t)r * C + c];
      const float inv = 1.0f / fmaxf(nr, 1.0f);
      for (int d = 0; d < D; ++d) {
        kbar[((int64_t)r * C + c) * D + d] = f2bf(skr[c * D + d] * inv);
        vbar[((int64_t)r * C + c) * D + d] = f2bf(svr[c * D + d] * inv);
      }
      logn[(int64_t)r * C + c] = nr > 0.5f ? oro_logf(fmaxf(nr, 1.0f)) : -INFINITY;
    }
    free(skr);
    free(svr);
  }
}

/* OpenAttention.flash in double precision (the fp32 estimator of methods_eager.selftest :708-719):
 * softmax over valid tokens (q.k*sm) and proxies (q.kbar*sm + ln n) against their values.
 * prow_div = 1: proxies per query row; = G (BQ/BH): per KV head.  out: (BQ, D) double. */
void oro_flash(int BQ, int BH, int64_t Kdim, int n_sel, int n_exp, int NB, int prow_div, const uint16_t* q,
               const uint16_t* k, const uint16_t* v, const int32_t* sel, const int32_t* exp_idx,
               const uint16_t* kbar, const uint16_t* vbar, const float* logn, double sm_scale, double* out) {
  const int Gq = BQ / BH;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < BQ; ++r) {
    const int kvh = r / Gq;
    const int prow = r / prow_div;
    double qd[D];
    for (int d = 0; d < D; ++d) qd[d] = bf2f(q[(int64_t)r * D + d]);
    const int tot = n_sel + n_exp + NB;
    double* z = (double*)malloc(sizeof(double) * (tot > 0 ? tot : 1));
    double m = -INFINITY;
    for (int j = 0; j < tot; ++j) {
      z[j] = -INFINITY;
      if (j < n_sel + n_exp) {
        int t = j < n_sel ? sel[(int64_t)r * n_sel + j] : exp_idx[(int64_t)r * n_exp + j - n_sel];
        if (t < 0 || t >= Kdim) continue;
        const uint16_t* kr = k + ((int64_t)kvh * Kdim + t) * D;
        double dot = 0;
        for (int d = 0; d < D; ++d) dot += qd[d] * (double)bf2f(kr[d]);
        z[j] = dot * sm_scale;
      } else {
        int b = j - n_sel - n_exp;
        double ln = logn[(int64_t)r * NB + b];
        if (ln == -INFINITY) continue;
        const uint16_t* kr = kbar + ((int64_t)prow * NB + b) * D;
        double dot = 0;
        for (int d = 0; d < D; ++d) dot += qd[d] * (double)bf2f(kr[d]);
        z[j] = dot * sm_scale + ln;
      }
      if (z[j] > m) m = z[j];
    }
    double l = 0, acc[D];
    for (int d = 0; d < D; ++d) acc[d] = 0;
    if (m > -INFINITY) {
      for (int j = 0; j < tot; ++j) {
        if (z[j] == -INFINITY) continue;
        double p = exp(z[j] - m);
        l += p;
        const uint16_t* vr;
        if (j < n_sel + n_exp) {
          int t = j < n_sel ? sel[(int64_t)r * n_sel + j] : exp_idx[(int64_t)r * n_exp + j - n_sel];
          vr = v + ((int64_t)kvh * Kdim + t) * D;
        } else {
          vr = vbar + ((int64_t)prow * NB + (j - n_sel - n_exp)) * D;
        }
        for (int d = 0; d < D; ++d) acc[d] += p * (double)bf2f(vr[d]);
      }
    }
    for (int d = 0; d < D; ++d) out[(int64_t)r * D + d] = l > 0 ? acc[d] / l : 0.0;
    free(z);
  }
}

/* ------------------------------------------------------------------ per-request build */
/* QGS codes of one request: z[h,t,j] = sum_d k.U (d ascending, fmaf), scale_j = max(amax_t |z| / 127,
 * 1e-12), code = clamp(rint(z / scale), +-127).  (methods_eager.py:520-524, ours_fastbuild.py:257-260)
 * K: (8, Lmax, D) bf16 of the request, U: (8, D, 32), scale: (8, 32), codes: (8, Lmax, 32). */
void oro_build_codes(int T, int Lmax, const uint16_t* K, const float* U, float* scale, int8_t* codes) {
#pragma omp parallel for schedule(static)
  for (int h = 0; h < HKV; ++h) {
    float* z = (float*)malloc(sizeof(float) * (size_t)T * RQ);
    const float* Uh = U + (int64_t)h * D * RQ;
    float amax[RQ];
    for (int j = 0; j < RQ; ++j) amax[j] = 0.0f;
    for (int t = 0; t < T; ++t) {
      const uint16_t* kr = K + ((int64_t)h * Lmax + t) * D;
      float kf[D];
      for (int d = 0; d < D; ++d) kf[d] = bf2f(kr[d]);
      for (int j = 0; j < RQ; ++j) {
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc = fmaf(kf[d], Uh[d * RQ + j], acc);
        z[(int64_t)t * RQ + j] = acc;
        float a = fabsf(acc);
        if (a > amax[j]) amax[j] = a;
      }
    }
    for (int j = 0; j < RQ; ++j) scale[h * RQ + j] = fmaxf(amax[j] / 127.0f, 1e-12f);
    for (int t = 0; t < T; ++t)
      for (int j = 0; j < RQ; ++j) {
        float c = rintf(z[(int64_t)t * RQ + j] / scale[h * RQ + j]);
        c = fminf(fmaxf(c, -127.0f), 127.0f);
        codes[((int64_t)h * Lmax + t) * RQ + j] = (int8_t)c;
      }
    free(z);
  }
}

/* QGC projection of one request: zp[h,t,c] = bf16(sum_d k.W (d ascending, fmaf)) per query head h
 * (K row h/4), colmean = (float)(sum_t zp / T) with the sum in double, sequential over tiles of 256
 * tokens; zP = zp - colmean.  (methods_eager.py:529-532)  W: (32, D, 16) bf16, zP: (32, T, 16). */
void oro_project(int T, int Lmax, const uint16_t* K, const uint16_t* W, float* zP, float* colmean) {
#pragma omp parallel for schedule(static)
  for (int h = 0; h < HQ; ++h) {
    const uint16_t* Wh = W + (int64_t)h * D * RC;
    float wf[D * RC];
    for (int i = 0; i < D * RC; ++i) wf[i] = bf2f(Wh[i]);
    double sum[RC];
    for (int c = 0; c < RC; ++c) sum[c] = 0.0;
    for (int t0 = 0; t0 < T; t0 += 256) {
      double part[RC];
      for (int c = 0; c < RC; ++c) part[c] = 0.0;
      for (int t = t0; t < T && t < t0 + 256; ++t) {
        const uint16_t* kr = K + ((int64_t)(h / G) * Lmax + t) * D;
        float kf[D];
        for (int d = 0; d < D; ++d) kf[d] = bf2f(kr[d]);
        for (int c = 0; c < RC; ++c) {
          float acc = 0.0f;
          for (int d = 0; d < D; ++d) acc = fmaf(kf[d], wf[d * RC + c], acc);
          float zb = bfr(acc);
          zP[((int64_t)h * T + t) * RC + c] = zb;
          part[c] = part[c] + (double)zb;
        }
      }
      for (int c = 0; c < RC; ++c) sum[c] = sum[c] + part[c];
    }
    for (int c = 0; c < RC; ++c) colmean[h * RC + c] = (float)(sum[c] / (double)T);
    for (int t = 0; t < T; ++t)
      for (int c = 0; c < RC; ++c) {
        float* p = &zP[((int64_t)h * T + t) * RC + c];
        *p = *p - colmean[h * RC + c];
      }
  }
}

/* One Lloyd assignment for all 32 query heads of a request: dist = bf16(bf16(zb.cb) - half),
 * zb = bf16(zP), cb = bf16(cent), half = bf16(0.5 * sum_c cent_c^2); argmax, ties -> lower id.
 * (methods_eager.py:538-542, ours_fastbuild.py:52-82) */
void oro_kmeans_assign(int T, int C, const float* zP, const float* cent, int32_t* asg, int64_t asg_stride) {
#pragma omp parallel for schedule(static)
  for (int h = 0; h < HQ; ++h) {
    float* cb = (float*)malloc(sizeof(float) * C * RC);
    float* half = (float*)malloc(sizeof(float) * C);
    for (int i = 0; i < C; ++i) {
      float nrm = 0.0f;
      for (int c = 0; c < RC; ++c) {
        const float x = cent[((int64_t)h * C + i) * RC + c];
        cb[i * RC + c] = bfr(x);
        float xx = x * x;
        nrm = nrm + xx;
      }
      half[i] = bfr(0.5f * nrm);
    }
    for (int t = 0; t < T; ++t) {
      float zb[RC];
      for (int c = 0; c < RC; ++c) zb[c] = bfr(zP[((int64_t)h * T + t) * RC + c]);
      int best = 0;
      float bestv = -INFINITY;
      for (int i = 0; i < C; ++i) {
        float acc = 0.0f;
        for (int c = 0; c < RC; ++c) acc = fmaf(zb[c], cb[i * RC + c], acc);
        float dd = bfr(bfr(acc) - half[i]);
        if (dd > bestv) {
          bestv = dd;
          best = i;
        }
      }
      asg[(int64_t)h * asg_stride + t] = best;
    }
    free(cb);
    free(half);
  }
}

/* Lloyd update: cent_i = (sum of member zP in token order, fp32) / count; an empty cluster takes its
 * seed point zP[init_i].  nb = member counts.  (methods_eager.py:543-545) */
void oro_kmeans_update(int T, int C, const float* zP, const int32_t* asg, int64_t asg_stride, const int64_t* init,
                       float* cent, float* nb) {
#pragma omp parallel for schedule(static)
  for (int h = 0; h < HQ; ++h) {
    float* acc = (float*)calloc((size_t)C * RC, sizeof(float));
    float* cnt = (float*)calloc((size_t)C, sizeof(float));
    for (int t = 0; t < T; ++t) {
      const int a = asg[(int64_t)h * asg_stride + t];
      for (int c = 0; c < RC; ++c) acc[a * RC + c] = acc[a * RC + c] + zP[((int64_t)h * T + t) * RC + c];
      cnt[a] = cnt[a] + 1.0f;
    }
    for (int i = 0; i < C; ++i) {
      for (int c = 0; c < RC; ++c) {
        float v = cnt[i] > 0.0f ? acc[i * RC + c] / fmaxf(cnt[i], 1.0f) : zP[((int64_t)h * T + init[i]) * RC + c];
        cent[((int64_t)h * C + i) * RC + c] = v;
      }
      nb[(int64_t)h * C + i] = cnt[i];
    }
    free(acc);
    free(cnt);
  }
}

/* CSR member lists (stable by position) and per-cluster sums of k, k*k, v in member order, fp32
 * (ours_fused.py:436-445 + ours_fastbuild.py:111-139; = the scatter_add sums of methods_eager.py:549-555).
 * mem: (32, Lmax) first T used; cstart, clen: (32, C); Sk, Sk2, Sv: (32, C, D). */
void oro_csr_sums(int T, int Lmax, int C, const uint16_t* K, const uint16_t* V, const int32_t* asg,
                  int64_t asg_stride, int32_t* mem, int32_t* cstart, int32_t* clen, float* Sk, float* Sk2,
                  float* Sv) {
#pragma omp parallel for schedule(static)
  for (int h = 0; h < HQ; ++h) {
    int32_t* cnt = (int32_t*)calloc((size_t)C, sizeof(int32_t));
    const int32_t* ar = asg + (int64_t)h * asg_stride;
    for (int t = 0; t < T; ++t) cnt[ar[t]]++;
    int run = 0;
    for (int i = 0; i < C; ++i) {
      cstart[h * C + i] = run;
      clen[h * C + i] = cnt[i];
      run += cnt[i];
      cnt[i] = 0;
    }
    for (int t = 0; t < T; ++t) {
      const int a = ar[t];
      mem[(int64_t)h * Lmax + cstart[h * C + a] + cnt[a]] = t;
      cnt[a]++;
    }
    for (int i = 0; i < C; ++i) {
      float* sk = Sk + ((int64_t)h * C + i) * D;
      float* sk2 = Sk2 + ((int64_t)h * C + i) * D;
      float* sv = Sv + ((int64_t)h * C + i) * D;
      for (int d = 0; d < D; ++d) sk[d] = sk2[d] = sv[d] = 0.0f;
      for (int j = 0; j < clen[h * C + i]; ++j) {
        const int t = mem[(int64_t)h * Lmax + cstart[h * C + i] + j];
        const uint16_t* kr = K + ((int64_t)(h / G) * Lmax + t) * D;
        const uint16_t* vr = V + ((int64_t)(h / G) * Lmax + t) * D;
        for (int d = 0; d < D; ++d) {
          float kf = bf2f(kr[d]);
          sk[d] = sk[d] + kf;
          float kk = kf * kf;
          sk2[d] = sk2[d] + kk;
          sv[d] = sv[d] + bf2f(vr[d]);
        }
      }
    }
    free(cnt);
  }
}
