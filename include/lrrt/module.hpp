// Module (a loaded sm_100a cubin/fatbin) and Kernel handles, following
// light-rocm-runtime include/lrrt/module.hpp:12-80.
#ifndef LRRT_MODULE_HPP_
#define LRRT_MODULE_HPP_

#include "lrrt/runtime.hpp"

#include <vector>

namespace lrrt {

using KernelProperties = lr_kernel_properties_t;

// Non-owning: kernels live as long as the module that produced them.
class Kernel {
public:
  explicit Kernel(lr_kernel_t *kernel) : kernel_(kernel) {}
  lr_kernel_t *get() const { return kernel_; }
  KernelProperties properties() const {
    KernelProperties value{};
    check(lr_kernel_get_properties(kernel_, &value), "lr_kernel_get_properties");
    return value;
  }

private:
  lr_kernel_t *kernel_;
};

class Module : public OwnedHandle<lr_module_t, lr_module_destroy> {
public:
  Module(lr_device_t device, const void *image, size_t image_size) {
    check(lr_module_load_hsaco(device, image, image_size, out()),
          "lr_module_load_hsaco");
  }
  Module(lr_device_t device, const std::vector<unsigned char> &image)
      : Module(device, image.data(), image.size()) {}
  Module(Device device, const void *image, size_t image_size)
      : Module(device.get(), image, image_size) {}
  Module(Device device, const std::vector<unsigned char> &image)
      : Module(device.get(), image.data(), image.size()) {}

  Kernel kernel(const char *name) const {
    lr_kernel_t *handle = nullptr;
    check(lr_kernel_get(get(), name, &handle), "lr_kernel_get");
    return Kernel(handle);
  }
};

} // namespace lrrt

#endif // LRRT_MODULE_HPP_
