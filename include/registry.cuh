// Interface of VibeGEMM's include/registry.cuh (AnonymousSC2026/VibeGEMM, GNU General Public
// License v3.0), kept identical so backends drop in; see NOTICE.
//
// KernelRegistry — static self-registration of GEMM backends.
//
// Same contract as the reference registry (include/registry.cuh:10-70 of VibeGEMM):
// backends register a factory with a priority from a static initialiser; make_all()
// instantiates them ordered by priority (stable), so cuBLAS (priority 0) comes first
// and serves as the engine's reference. Adds REGISTER_B200_KERNEL (priority 3).
// Translation units holding registrations must be linked whole-archive (or be part of
// a shared library), otherwise the linker drops the static registrar objects.
#pragma once

#include <algorithm>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "backend.cuh"

class KernelRegistry {
  public:
    using Factory = std::function<std::shared_ptr<GemmBackend>()>;

    static KernelRegistry &instance() {
        static KernelRegistry registry;
        return registry;
    }

    void add(int priority, const char *display_name, Factory factory) {
        items_.push_back(Item{priority, display_name, std::move(factory)});
    }

    // Fresh backend instances in priority order (ties keep registration order).
    std::vector<std::shared_ptr<GemmBackend>> make_all() const {
        std::vector<Item> ordered(items_);
        std::stable_sort(ordered.begin(), ordered.end(),
                         [](const Item &x, const Item &y) { return x.priority < y.priority; });
        std::vector<std::shared_ptr<GemmBackend>> backends;
        backends.reserve(ordered.size());
        for (const Item &it : ordered)
            backends.push_back(it.factory());
        return backends;
    }

    // Registered display names in priority order, without instantiating anything.
    std::vector<std::string> names() const {
        std::vector<Item> ordered(items_);
        std::stable_sort(ordered.begin(), ordered.end(),
                         [](const Item &x, const Item &y) { return x.priority < y.priority; });
        std::vector<std::string> out;
        for (const Item &it : ordered)
            out.emplace_back(it.name);
        return out;
    }

  private:
    KernelRegistry() = default;
    struct Item {
        int priority;
        const char *name;
        Factory factory;
    };
    std::vector<Item> items_;
};

struct KernelRegistrar {
    KernelRegistrar(int priority, const char *name, KernelRegistry::Factory factory) {
        KernelRegistry::instance().add(priority, name, std::move(factory));
    }
};

#define VG_KREG_CAT2(a, b) a##b
#define VG_KREG_CAT(a, b) VG_KREG_CAT2(a, b)

// Backend class constructed with its display name.
#define VG_KREG_NAMED(priority, dn, BC, uid)                                                      \
    static ::KernelRegistrar VG_KREG_CAT(vg_kreg_, uid)(                                           \
        priority, dn, []() -> std::shared_ptr<GemmBackend> { return std::make_shared<BC>(dn); })

// Backend class with a default constructor.
#define VG_KREG_PLAIN(priority, dn, BC, uid)                                                      \
    static ::KernelRegistrar VG_KREG_CAT(vg_kreg_, uid)(                                           \
        priority, dn, []() -> std::shared_ptr<GemmBackend> { return std::make_shared<BC>(); })

#define REGISTER_CUBLAS(dn, BC) VG_KREG_PLAIN(0, dn, BC, __COUNTER__)
#define REGISTER_A100_KERNEL(dn, BC) VG_KREG_NAMED(1, dn, BC, __COUNTER__)
#define REGISTER_H100_KERNEL(dn, BC) VG_KREG_NAMED(2, dn, BC, __COUNTER__)
#define REGISTER_B200_KERNEL(dn, BC) VG_KREG_NAMED(3, dn, BC, __COUNTER__)
