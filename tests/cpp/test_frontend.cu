// test_frontend.cu — the C++ API (include/choreo-ir/) exercised the way the
// reference's own unit and end-to-end tests exercise theirs
// (tests/test_shape.cpp, test_stride.cpp, test_layout.cpp, test_tensor.cpp,
// test_end2end.cpp, test_debug_cpu.cpp of the reference), plus the B200
// additions (swizzled shared-memory layouts, tile windows, auto_analyze,
// conv2d, batch/mixed-precision matmul).
//
// Groups starting with "cpu" need no GPU; "gpu" groups need a B200.
// Run: test_frontend cpu | gpu | all
#include <chrono>
#include <cmath>
#include <random>
#include <set>
#include <vector>

#include "choreo-ir/choreo-ir.hpp"
#include "choreo-ir/tensor/device_tile.hpp"
#include "choreo-ir/utils/profiler.hpp"
#include "mini_test.hpp"

using namespace choreo_ir;

// ======================================================================= CPU
TEST(cpu_shape, Constructors) {
  Shape s;
  EXPECT_EQ(s.ndims(), 0);
  EXPECT_TRUE(s.is_scalar());
  EXPECT_EQ(s.numel(), 1);
  Shape a({3, 4, 5});
  EXPECT_EQ(a.ndims(), 3);
  EXPECT_EQ(a[2], 5);
  EXPECT_EQ(a.numel(), 60);
  Shape v(std::vector<index_t>{2, 3, 4, 5});
  EXPECT_EQ(v.numel(), 120);
  index_t arr[3] = {6, 7, 8};
  Shape p(arr, 3);
  EXPECT_EQ(p.numel(), 336);
  EXPECT_EQ(make_shape(2, 3, 4).numel(), 24);
}

TEST(cpu_shape, AccessAndErrors) {
  Shape m({5, 8});
  EXPECT_EQ(m.at(1), 8);
  EXPECT_THROW(m[2], std::out_of_range);
  EXPECT_THROW(m.at(2), std::out_of_range);
  m[0] = 10;
  EXPECT_EQ(m.numel(), 80);
  EXPECT_EQ(Shape({10}).second_last_dim(), 1);
  EXPECT_EQ(Shape().last_dim(), 1);
  EXPECT_TRUE(Shape({3, 0, 4}).empty());
  EXPECT_THROW(Shape({5, 8}).reshape(Shape({3, 4})), std::invalid_argument);
  EXPECT_EQ(Shape({5, 8}).reshape(Shape({8, 5}))[0], 8);
  bool thrown = false;
  try {
    Shape too({1, 2, 3, 4, 5, 6, 7, 8, 9});
  } catch (const std::invalid_argument& e) {
    thrown = std::string(e.what()) == "Too many dimensions";
  }
  EXPECT_TRUE(thrown);
}

TEST(cpu_shape, TransposeSliceEquality) {
  Shape t = Shape({2, 3, 4}).transpose();
  EXPECT_EQ(t[0], 2);
  EXPECT_EQ(t[1], 4);
  EXPECT_EQ(t[2], 3);
  EXPECT_EQ(Shape().transpose().ndims(), 0);
  Shape s = Shape({2, 3, 4, 5}).slice(1, 3);
  EXPECT_EQ(s.ndims(), 2);
  EXPECT_EQ(s[0], 3);
  EXPECT_THROW(Shape({2, 3, 4, 5}).slice(3, 2), std::out_of_range);
  EXPECT_THROW(Shape({2, 3, 4, 5}).slice(0, 5), std::out_of_range);
  EXPECT_TRUE(Shape({5, 8}) == Shape({5, 8}));
  EXPECT_TRUE(Shape({5, 8}) != Shape({8, 5}));
  auto vec = Shape({2, 3, 4}).to_vector();
  EXPECT_EQ(vec.size(), 3u);
  EXPECT_EQ(Shape({1000, 1000, 1000}).numel(), 1000000000LL);
}

TEST(cpu_stride, RowColMajorOffsets) {
  Stride r = Stride::from_shape_row_major(Shape({2, 3, 4}));
  EXPECT_EQ(r[0], 12);
  EXPECT_EQ(r[1], 4);
  EXPECT_EQ(r[2], 1);
  Stride c = Stride::from_shape_col_major(Shape({2, 3, 4}));
  EXPECT_EQ(c[0], 1);
  EXPECT_EQ(c[1], 2);
  EXPECT_EQ(c[2], 6);
  EXPECT_EQ(r.offset(1, 2, 3), 12 + 8 + 3);
  EXPECT_EQ(r.offset(std::vector<index_t>{1, 2, 3}), 23);
  EXPECT_THROW(r.offset(1, 2), std::invalid_argument);
  EXPECT_TRUE(r.is_contiguous(Shape({2, 3, 4})));
  EXPECT_TRUE(c.is_contiguous_col_major(Shape({2, 3, 4})));
  EXPECT_FALSE(c.is_contiguous(Shape({2, 3, 4})));
  EXPECT_TRUE(r.is_coalesced());
  EXPECT_FALSE(c.is_coalesced());
  EXPECT_EQ(r.transpose()[1], 1);
  EXPECT_EQ(r.slice(1, 3)[0], 4);
  EXPECT_THROW(r.slice(2, 1), std::out_of_range);
  EXPECT_EQ(make_stride(8, 1)[0], 8);
}

TEST(cpu_layout, ReferenceBehaviour) {
  Layout d;
  EXPECT_EQ(d.ndims(), 0);
  EXPECT_EQ(d.numel(), 1);
  EXPECT_TRUE(d.layout_type() == LayoutType::ROW_MAJOR);
  Layout l(Shape({4, 6}));
  EXPECT_TRUE(l.is_contiguous());
  EXPECT_EQ(l.memory_size(DataType::FLOAT32), 96u);
  EXPECT_EQ(l.memory_size(DataType::FLOAT16), 48u);
  Layout cm(Shape({4, 6}), LayoutType::COLUMN_MAJOR);
  EXPECT_TRUE(cm.is_contiguous());
  EXPECT_EQ(l.offset(1, 2), 1 * 6 + 2);
  EXPECT_EQ(cm.offset(1, 2), 2 * 4 + 1);
  EXPECT_THROW(Layout(Shape({4, 6}), Stride({1})), std::invalid_argument);
  EXPECT_EQ(l.transpose().shape()[0], 6);
  EXPECT_EQ(l.reshape(Shape({6, 4})).shape()[0], 6);
  EXPECT_THROW(l.transpose().reshape(Shape({24})), std::runtime_error);
  EXPECT_THROW(l.reshape(Shape({5, 5})), std::invalid_argument);
  EXPECT_EQ(Layout(Shape({2, 3, 4})).slice(1, 3).shape()[0], 3);
  // tile(Shape) returns the layout itself (reference tests/test_layout.cpp:168-177)
  EXPECT_TRUE(l.tile(Shape({2, 2})).shape() == l.shape());
  EXPECT_THROW(l.tile(Shape({2})), std::invalid_argument);
  EXPECT_TRUE(Layout(Shape({32, 32})).is_tensor_core_compatible());
  EXPECT_FALSE(Layout(Shape({15, 17})).is_tensor_core_compatible());
  EXPECT_FALSE(Layout(Shape({32})).is_tensor_core_compatible());
  dim3 b = Layout(Shape({4, 6})).get_optimal_block_size();
  EXPECT_LE(b.x, 32u);
  dim3 g = Layout(Shape({4, 6})).get_grid_size();
  EXPECT_GE(g.x * b.x, 6u);
  EXPECT_GE(g.y * b.y, 4u);
  EXPECT_EQ(Layout().get_optimal_block_size().x, 1u);
  EXPECT_TRUE(make_row_major_layout(Shape({3, 3})) == Layout(Shape({3, 3})));
  EXPECT_FALSE(Layout(Shape({3, 4}), Stride({8, 2})).is_coalesced());
}

TEST(cpu_layout, Windows) {
  Layout l(Shape({10, 20}));
  Layout w = l.window({8, 16}, Shape({4, 8}));
  EXPECT_EQ(w.shape()[0], 2);  // clipped at the edge
  EXPECT_EQ(w.shape()[1], 4);
  EXPECT_EQ(w.stride()[0], 20);
  EXPECT_THROW(l.window({11, 0}, Shape({1, 1})), std::out_of_range);
  MatrixStrides m = matrix_strides(Shape({10, 20}), Stride({20, 1}));
  EXPECT_TRUE(m.valid && !m.transposed && m.ld == 20);
  MatrixStrides t = matrix_strides(Shape({20, 10}), Stride({1, 20}));
  EXPECT_TRUE(t.valid && t.transposed && t.ld == 20);
  EXPECT_FALSE(matrix_strides(Shape({4, 4}), Stride({2, 2})).valid);
  alignas(16) static char buf[64];
  EXPECT_TRUE(tma_addressable(buf, 8, 0, 1, 2));
  EXPECT_FALSE(tma_addressable(buf, 4097, 0, 1, 2));
  EXPECT_FALSE(tma_addressable(buf + 2, 8, 0, 1, 2));
}

TEST(cpu_smem, Swizzle128Layouts) {
  // within every 1024-byte atom the swizzle permutes 16-byte chunks
  std::set<uint32_t> seen;
  for (uint32_t row = 0; row < 8; ++row)
    for (uint32_t chunk = 0; chunk < 8; ++chunk) {
      const uint32_t off = SmemTileLayout::swizzle_128b(row * 128 + chunk * 16);
      EXPECT_EQ(off / 128, row);
      EXPECT_EQ((off / 16) % 8, chunk ^ row);
      seen.insert(off);
    }
  EXPECT_EQ(seen.size(), 64u);
  SmemTileLayout k{OperandMajor::K, 128, 1, 2, Swizzle::B128};
  EXPECT_EQ(k.bytes(), 16384);
  EXPECT_EQ(k.offset(0, 0), 0u);
  EXPECT_EQ(k.offset(1, 0), 128u + 16u);   // row 1, chunk 0 -> chunk 1
  EXPECT_EQ(k.offset(9, 8), 1024u + 128u + 0u);  // row 9 (atom 1, row 1), chunk 1 -> chunk 0
  EXPECT_EQ(k.lbo(), 16u);
  EXPECT_EQ(k.sbo(), 1024u);
  EXPECT_EQ(k.k_step_bytes(), 32u);
  SmemTileLayout mn{OperandMajor::MN, 64, 4, 2, Swizzle::B128};
  EXPECT_EQ(mn.bytes(), 32768);
  EXPECT_EQ(mn.lbo(), 8192u);
  EXPECT_EQ(mn.k_step_bytes(), 2048u);
  EXPECT_EQ(mn.offset(64, 0), 8192u);  // second MN chunk
  EXPECT_EQ(mn.offset(8, 1), 128u);  // K row 1, MN chunk 1 -> chunk 1 ^ 1 = 0
}

TEST(cpu_tensor, HostTensorsAndTransfers) {
  auto z = Tensor<float>::zeros(Shape({4, 5}), MemoryType::HOST);
  EXPECT_EQ(z.memory_type(), MemoryType::HOST);
  EXPECT_EQ(z.data()[7], 0.0f);
  auto o = Tensor<float>::ones(Shape({4, 5}), MemoryType::HOST);
  EXPECT_EQ(o(3, 4), 1.0f);
  o.fill(42.0f);
  EXPECT_EQ(o.data()[0], 42.0f);
  Tensor<float> copy = o;
  EXPECT_EQ(copy.data()[19], 42.0f);
  EXPECT_NE(copy.data(), o.data());
  Tensor<float> moved = std::move(copy);
  EXPECT_EQ(moved.data()[0], 42.0f);
  auto h = moved.to_host();
  EXPECT_EQ(h.data()[5], 42.0f);
  auto r1 = host_tensor<half>::random({16, 8});
  auto r2 = host_tensor<half>::random({16, 8});
  bool same = true, in_range = true;
  for (index_t i = 0; i < r1.numel(); ++i) {
    same = same && __half2float(r1.data()[i]) == __half2float(r2.data()[i]);
    const float v = __half2float(r1.data()[i]);
    in_range = in_range && v >= -1.0f && v <= 1.0f;
  }
  EXPECT_TRUE(same);
  EXPECT_TRUE(in_range);
  auto view = o.tile({1, 2}, Shape({2, 2}));
  EXPECT_EQ(view.data(), o.data() + 7);
  EXPECT_EQ(view.shape()[1], 2);
}

TEST(cpu_matmul, HostIdentityKAT) {
  // tests/test_debug_cpu.cpp:23-29 of the reference
  auto A = Tensor<float>::zeros(Shape({2, 2}), MemoryType::HOST);
  auto B = Tensor<float>::zeros(Shape({2, 2}), MemoryType::HOST);
  std::vector<float> a = {1, 2, 3, 4}, b = {1, 0, 0, 1};
  A.copy_from_host(a.data());
  B.copy_from_host(b.data());
  auto C = A * B;
  std::vector<float> c(4);
  C.copy_to_host(c.data());
  EXPECT_EQ(c[0], 1.0f);
  EXPECT_EQ(c[1], 2.0f);
  EXPECT_EQ(c[2], 3.0f);
  EXPECT_EQ(c[3], 4.0f);
}

TEST(cpu_matmul, HostHalfAccumulatesInHalf) {
  auto A = host_tensor<half>::random({8, 64}, -1, 1, 1);
  auto B = host_tensor<half>::random({64, 8}, -1, 1, 2);
  auto C = A * B;
  for (index_t i = 0; i < 8; ++i)
    for (index_t j = 0; j < 8; ++j) {
      half acc = __float2half(0.0f);
      for (index_t k = 0; k < 64; ++k)
        acc = __float2half(__half2float(acc) + __half2float(A(i, k)) * __half2float(B(k, j)));
      EXPECT_EQ(__half_as_ushort(C(i, j)), __half_as_ushort(acc));
    }
}

TEST(cpu_matmul, ErrorHandling) {
  // tests/test_end2end.cpp:342-352 of the reference
  auto A = Tensor<float>::zeros(Shape({64, 32}), MemoryType::HOST);
  auto B = Tensor<float>::zeros(Shape({64, 32}), MemoryType::HOST);
  EXPECT_THROW(A * B, std::runtime_error);
  auto C = Tensor<float>::zeros(Shape({32, 64}), MemoryType::HOST);
  EXPECT_THROW(A + C, std::runtime_error);
  try {
    auto X = A * B;
  } catch (const compute::ValidationError& e) {
    EXPECT_TRUE(std::string(e.what()).find("Matrix dimension mismatch: A(64x32) * B(64x32)") != std::string::npos);
  }
}

TEST(cpu_elementwise, HostReluAddConv) {
  auto x = host_tensor<float>::random({64, 32}, -2, 2, 3);
  auto y = relu(x);
  for (index_t i = 0; i < x.numel(); ++i) EXPECT_EQ(y.data()[i], std::max(x.data()[i], 0.0f));
  auto s = x + y;
  EXPECT_EQ(s.data()[5], x.data()[5] + y.data()[5]);
  auto in = host_tensor<half>::random({1, 5, 5, 8}, 0, 1, 4);
  auto w = host_tensor<half>::random({4, 3, 3, 8}, -0.2f, 0.2f, 5);
  auto out = conv2d(in, w, 1, 1);
  EXPECT_TRUE(out.shape() == Shape({1, 5, 5, 4}));
}

TEST(cpu_profiler, FlopFormulas) {
  EXPECT_NEAR(utils::calculate_matmul_tflops(8192, 8192, 8192, 1.0), 1099.511627776, 1e-6);
  EXPECT_NEAR(utils::calculate_conv_tflops(32, 256, 56, 56, 256, 3, 3, 1.0), 118.380036096, 1e-6);
}

// ======================================================================= GPU
namespace {
template <typename T>
std::vector<float> host_floats(const Tensor<T>& t) {
  std::vector<T> h(static_cast<size_t>(t.numel()));
  t.copy_to_host(h.data());
  std::vector<float> f(h.size());
  for (size_t i = 0; i < h.size(); ++i) f[i] = to_float(h[i]);
  return f;
}
// max |y - r| / max(|r|, 1e-3 * rms(r)) against an fp64 loop over the rounded inputs
template <typename T>
double rel_err_vs_f64(const Tensor<T>& A, const Tensor<T>& B, const std::vector<float>& y, bool ta = false) {
  const auto a = host_floats(A), b = host_floats(B);
  const index_t M = ta ? A.shape()[1] : A.shape()[0], K = ta ? A.shape()[0] : A.shape()[1], N = B.shape()[1];
  std::vector<double> r(static_cast<size_t>(M * N));
  double ss = 0;
  for (index_t i = 0; i < M; ++i)
    for (index_t j = 0; j < N; ++j) {
      double s = 0;
      for (index_t k = 0; k < K; ++k) s += double(ta ? a[k * M + i] : a[i * K + k]) * double(b[k * N + j]);
      r[i * N + j] = s;
      ss += s * s;
    }
  const double tau = 1e-3 * std::sqrt(ss / double(r.size()));
  double worst = 0;
  for (size_t i = 0; i < r.size(); ++i) worst = std::max(worst, std::fabs(y[i] - r[i]) / std::max(std::fabs(r[i]), tau));
  return worst;
}
}  // namespace

TEST(gpu_device, InitializeAndInfo) {
  EXPECT_TRUE(initialize());
  EXPECT_GE(device::get_device_count(), 1);
  EXPECT_TRUE(device::get_compute_capability() == ComputeCapability::SM_100);
  EXPECT_TRUE(device::is_tensor_core_supported());
  const auto& info = device::get_device_info();
  EXPECT_GE(info.multiprocessor_count, 100);
  EXPECT_GE(info.max_shared_memory_per_block, 200 * 1024);
  EXPECT_THROW(device::get_device_info(999), std::runtime_error);
}

TEST(gpu_tensor, DeviceFillCopyTransfer) {
  initialize();
  auto z = Tensor<float>::zeros(Shape({64, 32}));
  auto o = Tensor<half>::ones(Shape({64, 32}));
  EXPECT_EQ(host_floats(z)[0], 0.0f);
  EXPECT_EQ(host_floats(o)[2047], 1.0f);
  auto d = Tensor<float>::device(Shape({1024, 1024}));
  auto h = Tensor<float>::host(Shape({1024, 1024}));
  h.fill(42.0f);
  d.copy_from_host(h.data());
  EXPECT_EQ(host_floats(d)[12345], 42.0f);
  d.fill(7.0f);
  EXPECT_EQ(host_floats(d.to_host())[999999], 7.0f);
}

TEST(gpu_matmul, HalfBf16FloatAgainstFp64) {
  initialize();
  auto A = host_tensor<half>::random({256, 320}, -1, 1, 11).to_device();
  auto B = host_tensor<half>::random({320, 192}, -1, 1, 12).to_device();
  auto C = A * B;
  EXPECT_TRUE(C.memory_type() == MemoryType::DEVICE);
  EXPECT_LE(rel_err_vs_f64(A, B, host_floats(C)), 1e-2);
  auto Ab = host_tensor<bfloat16_t>::random({129, 100}, -1, 1, 13).to_device();
  auto Bb = host_tensor<bfloat16_t>::random({100, 77}, -1, 1, 14).to_device();
  EXPECT_LE(rel_err_vs_f64(Ab, Bb, host_floats(Ab * Bb)), 1e-2);
  auto Af = host_tensor<float>::random({70, 50}, -1, 1, 15).to_device();
  auto Bf = host_tensor<float>::random({50, 30}, -1, 1, 16).to_device();
  EXPECT_LE(rel_err_vs_f64(Af, Bf, host_floats(Af * Bf)), 1e-4);
}

TEST(gpu_matmul, TransposeViewsWindowsAndEpilogue) {
  initialize();
  auto At = host_tensor<half>::random({96, 160}, -1, 1, 21).to_device();  // stored K x M
  auto B = host_tensor<half>::random({96, 64}, -1, 1, 22).to_device();
  auto C = device_tensor<half>::zeros({160, 64});
  compute::matmul(At.transpose(), B.view(), C.view());
  EXPECT_LE(rel_err_vs_f64(At, B, host_floats(C), /*ta=*/true), 1e-2);
  // window of a larger C
  auto big = device_tensor<float>::zeros({300, 200});
  auto A2 = host_tensor<half>::random({100, 96}, -1, 1, 23).to_device();
  auto B2 = host_tensor<half>::random({96, 50}, -1, 1, 24).to_device();
  compute::matmul(A2.view(), B2.view(), big.tile({100, 100}, Shape({100, 50})));
  auto hb = host_floats(big);
  std::vector<float> win;
  for (int i = 0; i < 100; ++i)
    for (int j = 0; j < 50; ++j) win.push_back(hb[(100 + i) * 200 + 100 + j]);
  EXPECT_LE(rel_err_vs_f64(A2, B2, win), 1e-2);
  EXPECT_EQ(hb[0], 0.0f);
  EXPECT_EQ(hb[99 * 200 + 100], 0.0f);
  // alpha / beta / bias / relu
  auto A3 = host_tensor<half>::random({128, 64}, -1, 1, 25).to_device();
  auto B3 = host_tensor<half>::random({64, 128}, -1, 1, 26).to_device();
  auto C3 = device_tensor<half>::ones({128, 128});
  auto bias = device_tensor<float>::ones({128});
  compute::GEMMConfig cfg;
  cfg.bias = bias.data();
  cfg.bias_dtype = DataType::FLOAT32;
  cfg.relu = true;
  compute::gemm(A3, B3, C3, __float2half(2.0f), __float2half(0.5f), cfg);
  auto a3 = host_floats(A3), b3 = host_floats(B3), c3 = host_floats(C3);
  double worst = 0;
  for (int i = 0; i < 128; ++i)
    for (int j = 0; j < 128; ++j) {
      double s = 0;
      for (int k = 0; k < 64; ++k) s += double(a3[i * 64 + k]) * b3[k * 128 + j];
      const double want = std::max(0.0, 2.0 * s + 0.5 + 1.0);
      worst = std::max(worst, std::fabs(c3[i * 128 + j] - want) / std::max(std::fabs(want), 0.05));
    }
  EXPECT_LE(worst, 1e-2);
}

TEST(gpu_matmul, BatchMixedAndAccumulate) {
  initialize();
  auto A = host_tensor<half>::random({4, 64, 48}, -1, 1, 31).to_device();
  auto B = host_tensor<half>::random({4, 48, 40}, -1, 1, 32).to_device();
  auto C = batch_matmul(A, B);
  EXPECT_TRUE(C.shape() == Shape({4, 64, 40}));
  auto hc = host_floats(C), ha = host_floats(A), hb = host_floats(B);
  double worst = 0;
  for (int b = 0; b < 4; ++b)
    for (int i = 0; i < 64; ++i)
      for (int j = 0; j < 40; ++j) {
        double s = 0;
        for (int k = 0; k < 48; ++k) s += double(ha[(b * 64 + i) * 48 + k]) * hb[(b * 48 + k) * 40 + j];
        worst = std::max(worst, std::fabs(hc[(b * 64 + i) * 40 + j] - s) / std::max(std::fabs(s), 0.05));
      }
  EXPECT_LE(worst, 1e-2);
  // f16 inputs, f32 output
  auto A2 = host_tensor<half>::random({64, 48}, -1, 1, 33).to_device();
  auto B2 = host_tensor<half>::random({48, 32}, -1, 1, 34).to_device();
  auto C2 = device_tensor<float>::zeros({64, 32});
  matmul(A2, B2, C2);
  EXPECT_LE(rel_err_vs_f64(A2, B2, host_floats(C2)), 1e-4);
  // C += A * B
  auto C3 = A2 * B2;
  auto once = host_floats(C3);
  C3 += A2 * B2;
  auto twice = host_floats(C3);
  double w2 = 0;
  for (size_t i = 0; i < once.size(); ++i) w2 = std::max(w2, double(std::fabs(twice[i] - 2 * once[i])));
  EXPECT_LE(w2, 1e-2);
}

TEST(gpu_matmul, ErrorHandlingAndShapes) {
  initialize();
  auto A = Tensor<float>::zeros(Shape({64, 32}));
  auto B = Tensor<float>::zeros(Shape({64, 32}));
  EXPECT_THROW(A * B, std::runtime_error);
  auto C = Tensor<float>::zeros(Shape({32, 64}));
  EXPECT_THROW(A + C, std::runtime_error);
  // RealWorldUsagePattern (tests/test_end2end.cpp:239-265)
  auto W1 = host_tensor<float>::random({512, 256}, 0, 1).to_device();
  auto W2 = host_tensor<float>::random({256, 128}, 0, 1).to_device();
  auto in = host_tensor<float>::random({32, 512}, 0, 1).to_device();
  auto out = (in * W1) * W2;
  EXPECT_EQ(out.shape()[0], 32);
  EXPECT_EQ(out.shape()[1], 128);
  auto large = host_tensor<half>::random({256, 512}, 0, 1).to_device();
  auto W1h = host_tensor<half>::random({512, 256}, 0, 1).to_device();
  EXPECT_EQ((large * W1h).shape()[0], 256);
  // mixed element types convert A to B's type first
  auto Af = host_tensor<float>::random({16, 16}, -1, 1).to_device();
  auto Bh = host_tensor<half>::random({16, 16}, -1, 1).to_device();
  EXPECT_TRUE((Af * Bh).dtype() == DataType::FLOAT16);
}

TEST(gpu_elementwise, ReluAddDevice) {
  initialize();
  auto x = host_tensor<float>::random({64, 32}, -2, 2, 42);
  auto xd = x.to_device();
  auto y = host_floats(relu(xd));
  for (index_t i = 0; i < x.numel(); ++i) EXPECT_EQ(y[i], std::max(x.data()[i], 0.0f));
  auto s = host_floats(xd + xd);
  EXPECT_EQ(s[7], x.data()[7] + x.data()[7]);
}

TEST(gpu_conv, Conv2dAgainstFp64) {
  initialize();
  auto in = host_tensor<half>::random({2, 10, 12, 64}, 0, 1, 51);
  auto w = host_tensor<half>::random({64, 3, 3, 64}, -0.05f, 0.05f, 52);
  auto out = conv2d(in.to_device(), w.to_device(), 1, 1);
  EXPECT_TRUE(out.shape() == Shape({2, 10, 12, 64}));
  const auto o = host_floats(out);
  std::vector<double> r(o.size());
  double ss = 0;
  for (int n = 0; n < 2; ++n)
    for (int p = 0; p < 10; ++p)
      for (int q = 0; q < 12; ++q)
        for (int k = 0; k < 64; ++k) {
          double s = 0;
          for (int rr = 0; rr < 3; ++rr)
            for (int ss2 = 0; ss2 < 3; ++ss2) {
              const int h = p - 1 + rr, ww = q - 1 + ss2;
              if (h < 0 || h >= 10 || ww < 0 || ww >= 12) continue;
              for (int c = 0; c < 64; ++c)
                s += double(__half2float(in(n, h, ww, c))) * double(__half2float(w(k, rr, ss2, c)));
            }
          r[((n * 10 + p) * 12 + q) * 64 + k] = s;
          ss += s * s;
        }
  const double tau = 1e-3 * std::sqrt(ss / r.size());
  double worst = 0;
  for (size_t i = 0; i < r.size(); ++i) worst = std::max(worst, std::fabs(o[i] - r[i]) / std::max(std::fabs(r[i]), tau));
  EXPECT_LE(worst, 1e-2);
}

TEST(gpu_host_pipeline, GemmAndConvOnHostTensors) {
  initialize();
  // GEMM: host A, B, bias -> host C through the pipelined host plan, with the
  // host buffers page-locked for the run; then B and bias resident on the device.
  auto A = host_tensor<bfloat16_t>::random({1100, 256}, -1, 1, 71);
  auto B = host_tensor<bfloat16_t>::random({256, 192}, -1, 1, 72);
  auto bias = host_tensor<bfloat16_t>::random({192}, -0.5f, 0.5f, 73);
  auto C = host_tensor<bfloat16_t>::zeros({1100, 192});
  {
    PinnedHost pa(A), pc(C);
    compute::HostGemmPlan<bfloat16_t> plan(1100, 192, 256, /*has_bias=*/true, /*relu=*/true, /*parts=*/3);
    EXPECT_EQ(plan.info().parts, 3);  // 367-row parts rounded up to 512-row tiles: 512, 512, 76
    plan.run(A, B, C, &bias);
    plan.synchronize();
    auto C2 = host_tensor<bfloat16_t>::zeros({1100, 192});
    auto Bd = B.to_device();
    auto biasd = bias.to_device();
    plan.run(A, Bd, C2, &biasd);
    plan.synchronize();
    for (index_t i = 0; i < C.numel(); ++i) EXPECT_EQ(to_float(C.data()[i]), to_float(C2.data()[i]));
  }
  double worst = 0, ss = 0;
  std::vector<double> r(1100 * 192);
  for (int i = 0; i < 1100; ++i)
    for (int j = 0; j < 192; ++j) {
      double s = to_float(bias(j));
      for (int k = 0; k < 256; ++k) s += double(to_float(A(i, k))) * double(to_float(B(k, j)));
      r[i * 192 + j] = s < 0 ? 0 : s;
      ss += s * s;
    }
  const double tau = 1e-3 * std::sqrt(ss / r.size());
  for (size_t i = 0; i < r.size(); ++i)
    worst = std::max(worst, std::fabs(to_float(C.data()[i]) - r[i]) / std::max(std::fabs(r[i]), tau));
  EXPECT_LE(worst, 1e-2);
  // conv: host activations and weights -> host output; equals the device conv2d.
  auto in = host_tensor<half>::random({3, 8, 9, 64}, 0, 1, 74);
  auto w = host_tensor<half>::random({64, 3, 3, 64}, -0.05f, 0.05f, 75);
  compute::HostConvPlan<half> cplan(in.shape(), w.shape(), 1, 1, false, false, 2);
  auto out = host_tensor<half>::zeros(cplan.output_shape());
  cplan.run(in, w, out);
  cplan.synchronize();
  auto ref = conv2d(in.to_device(), w.to_device(), 1, 1).to_host();
  for (index_t i = 0; i < out.numel(); ++i) EXPECT_EQ(to_float(out.data()[i]), to_float(ref.data()[i]));
  // contract: a device tensor where the plan streams host memory
  EXPECT_THROW(cplan.run(in.to_device(), w, out), std::runtime_error);
}

namespace {
__global__ void fill_grid_kernel(int* out, int value) {
  if (threadIdx.x == 0) out[blockIdx.x] = value;
}
}  // namespace

TEST(gpu_auto, AnalyzeAndLaunch) {
  initialize();
  auto A = device_tensor<half>::random({4096, 1024}, -1, 1, 61);
  auto B = device_tensor<half>::random({1024, 2048}, -1, 1, 62);
  auto C = device_tensor<half>::zeros({4096, 2048});
  auto cfg = auto_analyze(A, B, C);
  EXPECT_TRUE(cfg.use_tensor_cores);
  EXPECT_TRUE(cfg.tile_sizes.x == 128u || cfg.tile_sizes.x == 256u || cfg.tile_sizes.x == 512u);
  EXPECT_TRUE(cfg.cluster_m == (cfg.tile_sizes.x == 128u ? 1 : 2));
  EXPECT_EQ(cfg.block_dim.x, 320u);
  EXPECT_GE(cfg.shared_memory, 150u * 1024u);
  EXPECT_LE(cfg.grid_dim.x, 148u);
  cfg.launch();
  cudaDeviceSynchronize();
  EXPECT_EQ(choreo_sync_status(nullptr), 0);
  auto C2 = A * B;
  auto h1 = host_floats(C), h2 = host_floats(C2);
  EXPECT_TRUE(h1 == h2);
  // the analysed grid drives a caller's own kernel
  int* d = nullptr;
  cudaMalloc(&d, cfg.grid_dim.x * sizeof(int));
  LaunchConfig user = cfg;
  user.shared_memory = 0;
  user.block_dim = dim3(32);
  user.launch(fill_grid_kernel, d, 5);
  std::vector<int> h(cfg.grid_dim.x);
  cudaMemcpy(h.data(), d, h.size() * sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d);
  EXPECT_EQ(h.back(), 5);
  finalize();
}

// -------------------------------------------------- device-side tile movement
namespace {
constexpr int kTR = 32, kTC = 64;
using TileMap = device::TmaTileMap<half, kTR, kTC>;

// One CTA: the tile at (row0, col0) by `shared = global.tile(...)` and by a
// TMA tile load, both written out dense; the copied tile stored back into
// `back` at the same place.
__global__ void tile_move_kernel(device::GlobalMatrix<half> g, const __grid_constant__ TileMap tm, int row0,
                                 int col0, half* out_copy, half* out_tma, device::GlobalMatrix<half> back,
                                 int* flags) {
  __shared__ alignas(128) half s_copy[kTR * kTC];
  __shared__ alignas(128) half s_tma[kTR * kTC];
  __shared__ uint64_t mbar;
  __shared__ int issued;
  device::SharedTile<half, kTR, kTC> a(s_copy), b(s_tma);
  device::TileBarrier bar(&mbar);
  if (threadIdx.x == 0) bar.init(1);
  __syncthreads();
  a = g.tile(row0, col0);
  if (threadIdx.x == 0) issued = device::tma_load(tm, b, bar, row0, col0) ? 1 : 0;
  __syncthreads();
  const int ok = issued ? (bar.wait(0) ? 1 : 0) : 1;
  for (int i = threadIdx.x; i < kTR * kTC; i += blockDim.x) {
    out_copy[i] = s_copy[i];
    out_tma[i] = issued ? s_tma[i] : __float2half(-1.0f);
  }
  a.store(back.tile(row0, col0));
  if (threadIdx.x == 0) {
    flags[0] = issued;
    flags[1] = ok;
  }
}
}  // namespace

TEST(gpu_device_tile, SharedEqualsGlobalTileAndTma) {
  initialize();
  const int rows = 100, cols = 70, ld = 72;  // ragged matrix, 16-byte aligned rows
  std::vector<half> h(rows * ld);
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < ld; ++c) h[r * ld + c] = __float2half(c < cols ? static_cast<float>((r * cols + c) % 2048) : -7.0f);
  half *dg = nullptr, *dback = nullptr, *dcopy = nullptr, *dtma = nullptr;
  int* dflags = nullptr;
  cudaMalloc(&dg, h.size() * sizeof(half));
  cudaMalloc(&dback, h.size() * sizeof(half));
  cudaMalloc(&dcopy, kTR * kTC * sizeof(half));
  cudaMalloc(&dtma, kTR * kTC * sizeof(half));
  cudaMalloc(&dflags, 2 * sizeof(int));
  cudaMemcpy(dg, h.data(), h.size() * sizeof(half), cudaMemcpyHostToDevice);
  const device::GlobalMatrix<half> g{dg, rows, cols, ld};
  const device::GlobalMatrix<half> back{dback, rows, cols, ld};
  const TileMap tm = TileMap::make(g);
  struct Case { int row0, col0; bool tma; };
  const Case cases[] = {{0, 0, true}, {80, 40, true}, {16, 8, true}, {-8, -16, true}, {5, 3, false}, {99, 69, false}};
  for (const Case& cs : cases) {
    cudaMemset(dback, 0, h.size() * sizeof(half));
    tile_move_kernel<<<1, 128>>>(g, tm, cs.row0, cs.col0, dcopy, dtma, back, dflags);
    EXPECT_EQ(cudaDeviceSynchronize(), cudaSuccess);
    std::vector<half> copy(kTR * kTC), tma(kTR * kTC), bk(h.size());
    int flags[2];
    cudaMemcpy(copy.data(), dcopy, copy.size() * sizeof(half), cudaMemcpyDeviceToHost);
    cudaMemcpy(tma.data(), dtma, tma.size() * sizeof(half), cudaMemcpyDeviceToHost);
    cudaMemcpy(bk.data(), dback, bk.size() * sizeof(half), cudaMemcpyDeviceToHost);
    cudaMemcpy(flags, dflags, sizeof(flags), cudaMemcpyDeviceToHost);
    EXPECT_EQ(flags[0], cs.tma ? 1 : 0);  // unaligned innermost coordinate: no TMA issued
    EXPECT_EQ(flags[1], 1);
    int bad_copy = 0, bad_tma = 0;
    for (int r = 0; r < kTR; ++r)
      for (int c = 0; c < kTC; ++c) {
        const int gr = cs.row0 + r, gc = cs.col0 + c;
        const bool in = gr >= 0 && gr < rows && gc >= 0 && gc < cols;
        const float want = in ? static_cast<float>((gr * cols + gc) % 2048) : 0.0f;
        if (__half2float(copy[r * kTC + c]) != want) ++bad_copy;
        if (cs.tma && __half2float(tma[r * kTC + c]) != want) ++bad_tma;
      }
    EXPECT_EQ(bad_copy, 0);
    EXPECT_EQ(bad_tma, 0);
    int bad_back = 0;
    for (int r = 0; r < rows; ++r)
      for (int c = 0; c < ld; ++c) {
        const bool in_tile = r >= cs.row0 && r < cs.row0 + kTR && c >= cs.col0 && c < cs.col0 + kTC && c < cols;
        const float want = in_tile ? static_cast<float>((r * cols + c) % 2048) : 0.0f;
        if (__half2float(bk[r * ld + c]) != want) ++bad_back;
      }
    EXPECT_EQ(bad_back, 0);
  }
  cudaFree(dg);
  cudaFree(dback);
  cudaFree(dcopy);
  cudaFree(dtma);
  cudaFree(dflags);
  finalize();
}

TEST(cpu_device_tile, MapContractOnHost) {
  // the tensor-map contract is checked before any CUDA call
  alignas(64) unsigned char map[128];
  const int64_t dims[2] = {70, 100}, bad_strides[1] = {140};
  const uint32_t box[2] = {64, 32};
  EXPECT_EQ(choreo_tensor_map_encode(map, CHOREO_DTYPE_F16, 2, reinterpret_cast<void*>(0x10000), dims, bad_strides,
                                     box, 0),
            CHOREO_ERR_INVALID_ARG);
  const device::GlobalMatrix<half> g{reinterpret_cast<half*>(0x10002), 100, 70, 72};
  bool threw = false;
  try {
    (void)TileMap::make(g);  // base not 16-byte aligned
  } catch (const std::runtime_error&) {
    threw = true;
  }
  EXPECT_TRUE(threw);
}

int main(int argc, char** argv) { return mini_main(argc, argv); }
