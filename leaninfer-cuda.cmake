# LeanInfer B200 fused kernels: the leaninfer_cuda library target.
#
# Counterpart of the reference's cuda/leaninfer-cuda.cmake (:25-56), which a
# ggml build includes from its src/CMakeLists.txt:
#   include("<path>/leaninfer-cuda.cmake" OPTIONAL)
# and enables with  -DLEANINFER_CUDA=ON -DGGML_CUDA=ON.
# Same option, same target name, same link into `llama` when that target
# exists; the architecture is sm_100a only (B200), never inherited from the
# parent build, because the kernels use tcgen05, TMEM and TMA instructions
# that exist only there.
#
# LEANINFER_CUDA_SHARED=ON builds a shared library instead of the static one
# (the form the Python binding loads).

cmake_minimum_required(VERSION 3.24)

option(LEANINFER_CUDA "Enable LeanInfer CUDA fused kernels (B200, sm_100a)" OFF)
option(LEANINFER_CUDA_SHARED "Build leaninfer_cuda as a shared library" OFF)

if (LEANINFER_CUDA AND NOT GGML_CUDA)
    message(WARNING "LEANINFER_CUDA=ON requires -DGGML_CUDA=ON")
elseif (LEANINFER_CUDA)
    set(_LI_DIR "${CMAKE_CURRENT_LIST_DIR}")
    enable_language(CUDA)
    find_package(CUDAToolkit REQUIRED)

    file(GLOB _LI_SRC CONFIGURE_DEPENDS "${_LI_DIR}/leaninfer_b200/csrc/*.cu")
    if (LEANINFER_CUDA_SHARED)
        add_library(leaninfer_cuda SHARED ${_LI_SRC})
    else()
        add_library(leaninfer_cuda STATIC ${_LI_SRC})
    endif()

    set_target_properties(leaninfer_cuda PROPERTIES
        CUDA_ARCHITECTURES "100a-real"
        CUDA_STANDARD 17
        POSITION_INDEPENDENT_CODE ON
        CUDA_SEPARABLE_COMPILATION OFF)
    target_compile_options(leaninfer_cuda PRIVATE
        $<$<COMPILE_LANGUAGE:CUDA>:-lineinfo -diag-suppress=177>)
    # the real declarations of leaninfer-cuda.h (not its no-CUDA stubs)
    target_compile_definitions(leaninfer_cuda PUBLIC GGML_USE_CUDA)
    target_include_directories(leaninfer_cuda
        PUBLIC "${_LI_DIR}/include"
        PRIVATE "${_LI_DIR}/leaninfer_b200/csrc")
    target_link_libraries(leaninfer_cuda PUBLIC CUDA::cudart ${CMAKE_DL_LIBS})

    if (TARGET llama)
        target_link_libraries(llama PRIVATE leaninfer_cuda)
        target_compile_definitions(llama PUBLIC LEANINFER_CUDA)
        target_include_directories(llama PUBLIC "${_LI_DIR}/include")
    endif()
    message(STATUS "LeanInfer CUDA fused kernels ENABLED (sm_100a)")
endif()
