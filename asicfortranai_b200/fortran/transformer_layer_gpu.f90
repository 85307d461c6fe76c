! Drop-in replacement of module transformer_layer_gpu (transformer_layer_gpu.f90) over
! libq35.so.  Same public names.  init_gpu_layer uploads the layer's weights once (repacked
! on the GPU, where the whole layer then runs: RMSNorm, projections, RoPE, attention over
! the device KV cache, SwiGLU); apply_transformer_layer_gpu applies it; cleanup_gpu_layer
! releases every layer it uploaded.  Unlike the reference, whose module holds a single
! cached matrix, each TransformerLayer keeps its own device copy, so a model's 80 layers
! can all be initialised.  The layer argument of init_gpu_layer is intent(inout) here (it
! records the device handle).  Every procedure takes an optional stat=; without it a
! failure stops with libq35's message (q35_status).
! Compile after transformer_layer.f90.
module transformer_layer_gpu
    use iso_c_binding, only: c_int, c_ptr, c_null_ptr, c_associated
    use iso_fortran_env, only: int32, real32
    use q35_status, only: q35_check
    use q35_model_api, only: q35_model_destroy
    use transformer_layer
    implicit none
    private
    public :: init_gpu_layer, apply_transformer_layer_gpu
    public :: cleanup_gpu_layer

    logical, save :: gpu_initialized = .false.
    ! device layers made by init_gpu_layer, released together by cleanup_gpu_layer
    type(c_ptr), allocatable, save :: live(:)
    integer, save :: n_live = 0

contains

    logical function is_live(h)
        type(c_ptr), intent(in) :: h
        integer :: i
        is_live = .false.
        if (.not. c_associated(h)) return
        do i = 1, n_live
            if (c_associated(live(i), h)) then
                is_live = .true.
                return
            end if
        end do
    end function is_live

    subroutine remember(h)
        type(c_ptr), intent(in) :: h
        type(c_ptr), allocatable :: grown(:)
        if (.not. allocated(live)) allocate(live(16))
        if (n_live == size(live)) then
            allocate(grown(2 * size(live)))
            grown(1:n_live) = live(1:n_live)
            call move_alloc(grown, live)
        end if
        n_live = n_live + 1
        live(n_live) = h
    end subroutine remember

    ! transformer_layer_gpu.f90:35-105: the layer's matrices to the GPU (once)
    subroutine init_gpu_layer(layer, max_batch_size, stat)
        type(TransformerLayer), intent(inout), target :: layer
        integer(int32), intent(in) :: max_batch_size
        integer, intent(out), optional :: stat
        integer :: st
        if (present(stat)) stat = 0
        if (max_batch_size < 1) then
            if (present(stat)) then
                stat = 1
                return
            end if
            error stop "init_gpu_layer: max_batch_size must be positive"
        end if
        if (.not. is_live(layer%handle)) layer%handle = c_null_ptr   ! released by cleanup_gpu_layer
        if (.not. c_associated(layer%handle)) then
            call upload_layer(layer, st)
            if (st /= 0) then
                call q35_check(int(st, c_int), "init_gpu_layer", stat)
                return
            end if
            call remember(layer%handle)
        end if
        gpu_initialized = .true.
    end subroutine init_gpu_layer

    ! transformer_layer_gpu.f90:353-400
    subroutine apply_transformer_layer_gpu(layer, x, output, seq_len, stat)
        type(TransformerLayer), intent(inout), target :: layer
        integer(int32), intent(in), value :: seq_len
        real(real32), intent(in) :: x(seq_len, *)
        real(real32), intent(out) :: output(seq_len, *)
        integer, intent(out), optional :: stat
        if (present(stat)) stat = 0
        if (.not. gpu_initialized) then
            if (present(stat)) then
                stat = 6
                return
            end if
            error stop "apply_transformer_layer_gpu: call init_gpu_layer first"
        end if
        if (.not. is_live(layer%handle)) then
            call init_gpu_layer(layer, 1, stat)
            if (present(stat)) then
                if (stat /= 0) return
            end if
        end if
        call apply_transformer_layer(layer, x, output, seq_len, stat)
    end subroutine apply_transformer_layer_gpu

    ! transformer_layer_gpu.f90:110-121
    subroutine cleanup_gpu_layer()
        integer :: i
        integer(c_int) :: st
        do i = 1, n_live
            st = q35_model_destroy(live(i))
        end do
        n_live = 0
        gpu_initialized = .false.
    end subroutine cleanup_gpu_layer

end module transformer_layer_gpu
