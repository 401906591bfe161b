// Device check of lrrt::Bundle on a B200: loads the test bundle (manifest
// tests/cpp/bundle_manifest.json + the sm_100a cubin of bundle_kernels.cu,
// placed side by side by the build), packs kernargs through KernargBuffer and
// launches through every Bundle::launch overload. Usage:
//   bundle_device_test <manifest path>
#include "lrrt/bundle.hpp"

#include <cmath>
#include <cstdio>
#include <vector>

namespace {

int failures = 0;

void expect(bool condition, const char *what) {
  if (!condition) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    ++failures;
  }
}

} // namespace

int main(int argc, char **argv) {
  if (argc != 2) {
    std::fprintf(stderr, "usage: %s <manifest>\n", argv[0]);
    return 2;
  }
  try {
    lrrt::Runtime runtime;
    if (runtime.device_count() == 0) {
      std::fprintf(stderr, "no CUDA device\n");
      return 2;
    }
    lrrt::Device device = runtime.open_device(0);
    const lrrt::Bundle first(device, argv[1]); // first kernel of the manifest
    const lrrt::Bundle scale(device, argv[1], "scale");
    const lrrt::Bundle iota(device, argv[1], "iota");
    expect(first.manifest().name == "scale", "default kernel is the first one");

    const uint32_t n = 1000; // not a multiple of the block size
    std::vector<float> x(n), bias(n);
    for (uint32_t i = 0; i < n; ++i) {
      x[i] = 0.25f * static_cast<float>(i) - 7.0f;
      bias[i] = static_cast<float>(i % 13);
    }
    lrrt::DeviceBuffer x_device(device, n * sizeof(float));
    lrrt::DeviceBuffer bias_device(device, n * sizeof(float));
    lrrt::DeviceBuffer out_device(device, n * sizeof(float));
    lrrt::copy_to_device(x_device, x);
    lrrt::copy_to_device(bias_device, bias);

    // Optional bias left unbound -> null: out = 3x.
    lrrt::KernargBuffer args = scale.make_args();
    args.set("x", static_cast<const float *>(x_device.data()));
    args.set("out", static_cast<float *>(out_device.data()));
    args.set("factor", 3.0f);
    args.set("n", n);
    args.bind_optional_nulls();
    first.launch(n, args);
    device.synchronize();
    std::vector<float> out(n);
    lrrt::copy_to_host(out.data(), out_device, n * sizeof(float));
    bool exact = true;
    for (uint32_t i = 0; i < n; ++i) {
      exact = exact && out[i] == x[i] * 3.0f;
    }
    expect(exact, "scale without bias");

    // Bias bound, launched on an explicit queue after an event.
    lrrt::KernargBuffer with_bias = scale.make_args();
    with_bias.set(size_t{0}, static_cast<const float *>(x_device.data()));
    with_bias.set(size_t{1}, static_cast<float *>(out_device.data()));
    with_bias.set("bias", static_cast<const float *>(bias_device.data()));
    with_bias.set("factor", -0.5f);
    with_bias.set("n", n);
    lrrt::Queue queue(device.get());
    lrrt::Event ready(device.get());
    ready.record();
    scale.launch(queue, n, with_bias, {&ready});
    queue.synchronize();
    lrrt::copy_to_host(out.data(), out_device, n * sizeof(float));
    exact = true;
    for (uint32_t i = 0; i < n; ++i) {
      const float want = x[i] * -0.5f + bias[i];
      exact = exact && std::fabs(out[i] - want) <= 1e-6f * std::fmax(1.0f, std::fabs(want));
    }
    expect(exact, "scale with bias on a queue");

    // Second kernel of the bundle, default queue with a dependency list.
    const uint32_t m = 1537;
    lrrt::DeviceBuffer iota_device(device, m * sizeof(uint32_t));
    lrrt::KernargBuffer iota_args = iota.make_args();
    iota_args.set("out", static_cast<uint32_t *>(iota_device.data()));
    iota_args.set("offset", 100u);
    iota_args.set("n", m);
    lrrt::Event before(device.get());
    before.record();
    iota.launch(m, iota_args, {&before});
    device.synchronize();
    std::vector<uint32_t> values(m);
    lrrt::copy_to_host(values.data(), iota_device, m * sizeof(uint32_t));
    bool ordered = true;
    for (uint32_t i = 0; i < m; ++i) {
      ordered = ordered && values[i] == i + 100u;
    }
    expect(ordered, "iota kernel");
    expect(iota.launch_config(m).grid.x == 2048 && iota.launch_config(m).block.x == 256,
           "iota launch configuration");

    // A buffer for one kernel is refused by the other.
    expect([&] {
      try {
        iota.launch(m, args);
      } catch (const std::exception &) {
        return true;
      }
      return false;
    }(), "kernarg buffer of another kernel is rejected");
  } catch (const std::exception &error) {
    std::fprintf(stderr, "FAILED: %s\n", error.what());
    return 1;
  }
  if (failures == 0) {
    std::printf("bundle device checks: ok\n");
  }
  return failures == 0 ? 0 : 1;
}
