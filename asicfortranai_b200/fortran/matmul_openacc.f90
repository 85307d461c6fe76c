! Drop-in replacement of module matmul_openacc (matmul_openacc.f90) over libq35.so: the same
! two procedures and arguments, no OpenACC compiler needed.  The matrices stay resident on
! the GPU between calls with the same arrays (libq35's per-call cache).  Optional stat= as
! in the other drop-ins.  Compile after q35_status.f90.
module matmul_openacc
    use iso_c_binding, only: c_int, c_int8_t, c_int32_t, c_float
    use iso_fortran_env, only: int8, int32, real32
    use q35_status, only: q35_check
    implicit none
    private
    public :: matmul_int4_openacc, dequantize_output_openacc

    interface
        integer(c_int) function q35_matmul_int4_awq(A, W_Q, W_scales, C, M, N, K) &
                bind(C, name="q35_matmul_int4_awq")
            import :: c_int, c_int8_t, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N, K
            integer(c_int8_t), intent(in) :: A(*), W_Q(*)
            real(c_float), intent(in) :: W_scales(*)
            integer(c_int32_t), intent(inout) :: C(*)
        end function q35_matmul_int4_awq

        integer(c_int) function q35_dequantize_output(C, W_scales, Out, M, N) &
                bind(C, name="q35_dequantize_output")
            import :: c_int, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N
            integer(c_int32_t), intent(in) :: C(*)
            real(c_float), intent(in) :: W_scales(*)
            real(c_float), intent(inout) :: Out(*)
        end function q35_dequantize_output
    end interface

contains

    ! matmul_openacc.f90:30-73: int32 C(M,N)
    subroutine matmul_int4_openacc(A, W_Q, W_scales, C, M, N, K_dim, stat)
        integer(int8), intent(in) :: A(:,:)
        integer(int8), intent(in) :: W_Q(:,:)
        real(real32), intent(in) :: W_scales(:)
        integer(int32), intent(out) :: C(:,:)
        integer(int32), intent(in) :: M, N, K_dim
        integer, intent(out), optional :: stat
        call q35_check(q35_matmul_int4_awq(A, W_Q, W_scales, C, M, N, K_dim), "matmul_int4_openacc", stat)
    end subroutine matmul_int4_openacc

    ! matmul_openacc.f90:78-94: Out = real(C) * W_scales
    subroutine dequantize_output_openacc(C, W_scales, Out, M, N, stat)
        integer(int32), intent(in) :: C(:,:)
        real(real32), intent(in) :: W_scales(:)
        real(real32), intent(out) :: Out(:,:)
        integer(int32), intent(in) :: M, N
        integer, intent(out), optional :: stat
        call q35_check(q35_dequantize_output(C, W_scales, Out, M, N), "dequantize_output_openacc", stat)
    end subroutine dequantize_output_openacc

end module matmul_openacc
