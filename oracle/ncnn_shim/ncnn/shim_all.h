// shim_all.h -- CPU-only stand-in for the subset of the ncnn API that the
// reference's DiT host sources (src/dit_vk.cpp, src/awa_window.cpp,
// src/test_awa_unit.cpp) name.  TEST INFRASTRUCTURE: it exists only so that
// those reference files compile unchanged into oracle/_ref/ and serve as the
// parity checker; nothing in the product links it.
//
// What is real here:
//   * ncnn::Mat with the (w, h, data) constructor and float* decay
//     (ncnn mat.h semantics: dims=2, elemsize 4, external data not owned).
//   * ncnn::Net / ncnn::Extractor for one-layer "InnerProduct" graphs:
//     load_param_mem parses "0=num_output 1=bias_term 2=weight_data_size";
//     load_model(const unsigned char*) decodes the ncnn weight blob
//     [u32 tag][weights][fp32 bias], tag 0x01306B47 = fp16 weights,
//     tag 0 = fp32 weights (the layout reference export/ncnn_io.py writes);
//     extract() runs y = x W^T + b in fp32 (packed panels, AVX2/FMA 6x16
//     register micro-kernel, OpenMP) on a 2-D input.
// What is a stub: everything Vulkan (devices, allocators, pipelines,
// command buffers).  create_gpu_instance() reports failure, which is the
// state DitVk::init(use_cpu=true) expects.
#pragma once
#include <cstddef>
#include <cstring>   // ncnn mat.h pulls in <string.h>; reference sources rely on it
#include <cstdint>
#include <string>
#include <vector>
#include <memory>

namespace ncnn {

class Allocator;
class VkAllocator {
public:
    virtual ~VkAllocator() {}
    virtual void clear() {}
};
class VkBlobAllocator : public VkAllocator {};
class VkWeightAllocator : public VkAllocator {};

class VulkanDevice {
public:
    VkAllocator* acquire_blob_allocator() const { return nullptr; }
    VkAllocator* acquire_staging_allocator() const { return nullptr; }
};

int create_gpu_instance(int device_index = -1);
void destroy_gpu_instance();
VulkanDevice* get_gpu_device(int device_index = -1);
int get_gpu_count();

class Mat {
public:
    Mat() {}
    Mat(int _w, int _h, void* _data, size_t _elemsize = 4u, Allocator* = nullptr)
        : data(_data), elemsize(_elemsize), dims(2), w(_w), h(_h), d(1), c(1) {}
    void create(int _w, int _h, size_t _elemsize, Allocator* = nullptr) {
        owned = std::make_shared<std::vector<unsigned char>>((size_t)_w * _h * _elemsize);
        data = owned->data(); elemsize = _elemsize; dims = 2; w = _w; h = _h; d = 1; c = 1;
    }
    bool empty() const { return data == nullptr || (size_t)w * h * c == 0; }
    size_t total() const { return (size_t)w * h * d * c; }
    template <typename T> operator T*() { return (T*)data; }
    template <typename T> operator const T*() const { return (const T*)data; }

    std::shared_ptr<std::vector<unsigned char>> owned;
    void* data = nullptr;
    size_t elemsize = 0;
    int elempack = 1;
    int dims = 0, w = 0, h = 0, d = 0, c = 0;
};

class VkMat {
public:
    bool empty() const { return true; }
    size_t buffer_capacity() const { return 0; }
    int w = 0, h = 0, c = 0;
};

class Option {
public:
    bool use_vulkan_compute = false;
    bool use_fp16_arithmetic = false;
    bool use_fp16_storage = false;
    bool use_fp16_packed = false;
    bool use_bf16_storage = false;
    bool use_bf16_packed = false;
    bool use_packing_layout = false;
    int num_threads = 0;
    VkAllocator* blob_vkallocator = nullptr;
    VkAllocator* staging_vkallocator = nullptr;
    VkAllocator* workspace_vkallocator = nullptr;
};

class ParamDict {
public:
    int get(int, int def) const { return def; }
    float get(int, float def) const { return def; }
    std::string get(int, const std::string& def) const { return def; }
};

class ModelBin {
public:
    Mat load(int, int) const { return Mat(); }
};

class Pipeline;
class VkTransfer;
class VkCompute;

class Layer {
public:
    virtual ~Layer() {}
    virtual int load_param(const ParamDict&) { return 0; }
    virtual int load_model(const ModelBin&) { return 0; }
    virtual int create_pipeline(const Option&) { return 0; }
    virtual int destroy_pipeline(const Option&) { return 0; }
    virtual int upload_model(VkTransfer&, const Option&) { return 0; }
    virtual int forward(const std::vector<VkMat>&, std::vector<VkMat>&, VkCompute&, const Option&) const { return -1; }

    bool one_blob_only = false;
    bool support_inplace = false;
    bool support_vulkan = false;
    bool support_packing = false;
    bool support_bf16_storage = false;
    bool support_fp16_storage = false;
    std::string type;
    const VulkanDevice* vkdev = nullptr;
};

// One-layer InnerProduct network (the only graph shape DitVk::lin builds).
class Net;
class Extractor {
public:
    int input(const char* name, const Mat& in);
    int extract(const char* name, Mat& out);
private:
    friend class Net;
    explicit Extractor(const Net* n) : net(n) {}
    const Net* net;
    Mat in_;
};

class Net {
public:
    Net() {}
    ~Net() {}
    void set_vulkan_device(const VulkanDevice*) {}
    int load_param_mem(const char* mem);
    int load_model(const unsigned char* mem);
    Extractor create_extractor() const { return Extractor(this); }
    Option opt;

    // InnerProduct parameters and decoded weights (row-major W[out][in]).
    int num_output = 0, bias_term = 0, weight_data_size = 0;
    std::vector<float> weight;
    std::vector<float> bias;
};

}  // namespace ncnn
