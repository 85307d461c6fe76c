! Drop-in replacement of module matmul_cublas (matmul_cublas.f90) over libq35.so.  Same
! public names and arguments.  The reference dequantizes INT4 weights to fp32 and runs a
! cuBLAS SGEMM; here the packed codes stay packed on the GPU and the matmul is libq35's
! exact int32 kernel followed by the per-column dequant (Out = real(C) * scale,
! matmul_int4_groq.f90:58-69):
!   cublas_init / cublas_shutdown   the library context (shared with the model modules) /
!                                   release of the cached matrix
!   allocate_gpu_memory(M,N,K)      checks the sizes; the library sizes its buffers itself
!   dequantize_weights_gpu(W_Q,W_scales,N,K)   the matrix made resident (repacked once)
!   matmul_int4_cublas_cached(A,Out,M,N,K)     against that resident matrix
!   matmul_int4_cublas(A,W_Q,W_scales,Out,M,N,K)   per call; the library keeps the matrix
!                                   resident between calls with the same arrays
! Every procedure takes an optional stat=; without it a failure stops with libq35's
! message (q35_status).  Compile after q35_model_api.f90.
module matmul_cublas
    use iso_c_binding, only: c_int, c_int8_t, c_int32_t, c_float, c_ptr, c_null_ptr, c_associated, c_loc
    use iso_fortran_env, only: int8, int32, real32
    use q35_status, only: q35_check
    use q35_model_api, only: q35_fortran_context, q35_weights_upload, q35_weights_free, q35_matmul_cached, &
                             q35_matmul_int4_fused, Q35_FMT_INT4
    implicit none
    private
    public :: matmul_int4_cublas, matmul_int4_cublas_cached
    public :: cublas_init, cublas_shutdown
    public :: dequantize_weights_gpu, allocate_gpu_memory

    type(c_ptr), save :: cached_w = c_null_ptr          ! the resident matrix
    integer(int32), save :: cached_n = 0, cached_k = 0

contains

    ! matmul_cublas.f90:105-124
    subroutine cublas_init(stat)
        integer, intent(out), optional :: stat
        type(c_ptr) :: ctx
        ctx = q35_fortran_context(stat)
        if (c_associated(ctx)) print *, "libq35 initialized (B200, sm_100a)"
    end subroutine cublas_init

    ! matmul_cublas.f90:129-141
    subroutine cublas_shutdown()
        integer(c_int) :: st
        if (c_associated(cached_w)) then
            st = q35_weights_free(cached_w)
            cached_w = c_null_ptr
        end if
        cached_n = 0
        cached_k = 0
    end subroutine cublas_shutdown

    ! matmul_cublas.f90:146-170
    subroutine allocate_gpu_memory(M, N, K_dim, stat)
        integer(int32), intent(in) :: M, N, K_dim
        integer, intent(out), optional :: stat
        if (present(stat)) stat = 0
        if (M < 1 .or. N < 1 .or. K_dim < 2 .or. mod(K_dim, 2) /= 0) then
            if (present(stat)) then
                stat = 1
                return
            end if
            error stop "allocate_gpu_memory: M, N >= 1 and K_dim even >= 2"
        end if
    end subroutine allocate_gpu_memory

    ! matmul_cublas.f90:175-217: the INT4 matrix W_Q(K/2,N) made resident
    subroutine dequantize_weights_gpu(W_Q, W_scales, N, K_dim, stat)
        integer(int8), intent(in) :: W_Q(:,:)
        real(real32), intent(in) :: W_scales(:)
        integer(int32), intent(in) :: N, K_dim
        integer, intent(out), optional :: stat
        type(c_ptr) :: ctx
        integer :: st
        integer(c_int) :: fst
        ctx = q35_fortran_context(st)
        if (st /= 0) then
            call q35_check(int(st, c_int), "dequantize_weights_gpu", stat)
            return
        end if
        if (c_associated(cached_w)) then
            fst = q35_weights_free(cached_w)
            cached_w = c_null_ptr
        end if
        call q35_check(q35_weights_upload(ctx, Q35_FMT_INT4, W_Q, W_scales, c_null_ptr, N, K_dim, 0_c_int, cached_w), &
                       "dequantize_weights_gpu", stat)
        if (c_associated(cached_w)) then
            cached_n = N
            cached_k = K_dim
        end if
    end subroutine dequantize_weights_gpu

    ! matmul_cublas.f90:222-274: Out(M,N) = dequantized A x W_Q, W_Q passed on every call
    subroutine matmul_int4_cublas(A, W_Q, W_scales, Out, M, N, K_dim, stat)
        integer(int8), intent(in) :: A(:,:)
        integer(int8), intent(in) :: W_Q(:,:)
        real(real32), intent(in) :: W_scales(:)
        real(real32), intent(out) :: Out(:,:)
        integer(int32), intent(in) :: M, N, K_dim
        integer, intent(out), optional :: stat
        call q35_check(q35_matmul_int4_fused(A, W_Q, W_scales, Out, M, N, K_dim), "matmul_int4_cublas", stat)
    end subroutine matmul_int4_cublas

    ! matmul_cublas.f90:279-325: against the matrix of dequantize_weights_gpu
    subroutine matmul_int4_cublas_cached(A, Out, M, N, K_dim, stat)
        integer(int8), intent(in) :: A(:,:)
        real(real32), intent(out), target, contiguous :: Out(:,:)
        integer(int32), intent(in) :: M, N, K_dim
        integer, intent(out), optional :: stat
        type(c_ptr) :: ctx
        integer :: st
        if (present(stat)) stat = 0
        if (.not. c_associated(cached_w) .or. N /= cached_n .or. K_dim /= cached_k) then
            if (present(stat)) then
                stat = 6
                return
            end if
            error stop "matmul_int4_cublas_cached: no resident matrix of this shape (dequantize_weights_gpu first)"
        end if
        ctx = q35_fortran_context(st)
        call q35_check(q35_matmul_cached(ctx, cached_w, A, M, c_null_ptr, c_loc(Out)), "matmul_int4_cublas_cached", stat)
    end subroutine matmul_int4_cublas_cached

end module matmul_cublas
