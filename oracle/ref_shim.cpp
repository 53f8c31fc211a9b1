// ref_shim.cpp -- C entry points over the reference's own C++ CPU GEMM.
//
// TEST INFRASTRUCTURE ONLY.  Compiled together with the reference's
// int4_cube_lab/host/gemm_ref.cpp, straight from the reference source tree,
// by `make -C oracle ref` into oracle/_ref/ (never committed).  It only adapts
// raw pointers to the std::vector signatures declared in
// int4_cube_lab/host/gemm_ref.h:12-95, so ctypes can call:
//   ReferenceMidGroupGemm        (gemm_ref.cpp:199-240)
//   PackInt4Grouped              (gemm_ref.cpp:42-60)
//   SplitInt8ToInt4PlanesGrouped (gemm_ref.cpp:62-90)
//   WeightKSumPerGroup           (gemm_ref.cpp:129-152)
//   ActKSumNegPerGroup           (gemm_ref.cpp:181-197)
#include <cstdint>
#include <cstring>
#include <vector>

#include "gemm_ref.h"
#include "mg_kgeom.h"

extern "C" {

void ref_midgroup_gemm(const int8_t* a_q, const uint16_t* a_scale_g, const int8_t* w_q,
                       const uint16_t* w_scale_g, const uint16_t* w_zero_g, uint16_t* y,
                       uint32_t M, uint32_t N, uint32_t K, uint32_t gk, uint32_t mp)
{
    const uint32_t G = mgk::NumGroups(K, gk);
    const uint32_t Mp = mp ? mp : M;
    std::vector<int8_t> a(a_q, a_q + (size_t)M * K), w(w_q, w_q + (size_t)N * K);
    std::vector<uint16_t> as(a_scale_g, a_scale_g + (size_t)G * Mp);
    std::vector<uint16_t> ws(w_scale_g, w_scale_g + (size_t)G * N);
    std::vector<uint16_t> wz;
    if (w_zero_g) wz.assign(w_zero_g, w_zero_g + (size_t)G * N);
    std::vector<uint16_t> out;
    ReferenceMidGroupGemm(a, as, w, ws, wz, out, M, N, K, gk, mp);
    std::memcpy(y, out.data(), out.size() * sizeof(uint16_t));
}

void ref_pack_int4_grouped(const int8_t* v, uint32_t rows, uint32_t K, uint32_t gk, int8_t* out)
{
    std::vector<int8_t> in(v, v + (size_t)rows * K);
    std::vector<int8_t> p = PackInt4Grouped(in, rows, K, gk);
    std::memcpy(out, p.data(), p.size());
}

void ref_split_planes_grouped(const int8_t* a, uint32_t rows, uint32_t K, uint32_t gk,
                              int8_t* hi, int8_t* lo)
{
    std::vector<int8_t> in(a, a + (size_t)rows * K), h, l;
    SplitInt8ToInt4PlanesGrouped(in, rows, K, gk, h, l);
    std::memcpy(hi, h.data(), h.size());
    std::memcpy(lo, l.data(), l.size());
}

void ref_weight_ksum_per_group(const int8_t* w, uint32_t rows, uint32_t K, uint32_t gk,
                               int32_t* out)
{
    std::vector<int8_t> in(w, w + (size_t)rows * K);
    std::vector<int32_t> r = WeightKSumPerGroup(in, rows, K, gk);
    std::memcpy(out, r.data(), r.size() * sizeof(int32_t));
}

void ref_act_ksum_neg_per_group(const int8_t* a, uint32_t rows, uint32_t K, uint32_t gk,
                                int32_t* out)
{
    std::vector<int8_t> in(a, a + (size_t)rows * K);
    std::vector<int32_t> r = ActKSumNegPerGroup(in, rows, K, gk);
    std::memcpy(out, r.data(), r.size() * sizeof(int32_t));
}

}  // extern "C"
