! Status handling shared by the drop-in modules over libq35.so.  Every libq35 entry point
! returns an int status (0 = success) and keeps a message for the calling thread
! (q35_last_error).  q35_check gives a drop-in procedure the reference's behaviour -- a
! failure stops the program (the reference's error paths print and stop,
! matmul_cublas.f90:116-117) -- unless the caller passed the optional stat= argument,
! which then receives the status instead.
! Compile before the other modules: gfortran -c q35_status.f90
module q35_status
    use iso_c_binding, only: c_int, c_ptr, c_char, c_f_pointer, c_associated
    use iso_fortran_env, only: error_unit
    implicit none
    private
    public :: q35_check, q35_error_message

    interface
        type(c_ptr) function q35_last_error() bind(C, name="q35_last_error")
            import :: c_ptr
        end function q35_last_error
    end interface

contains

    subroutine q35_check(st, what, stat)
        integer(c_int), intent(in) :: st
        character(*), intent(in) :: what
        integer, intent(out), optional :: stat
        if (present(stat)) then
            stat = st
        else if (st /= 0) then
            write (error_unit, "(a)") what // ": " // q35_error_message()
            error stop 1
        end if
    end subroutine q35_check

    ! the calling thread's last libq35 message as a Fortran string
    function q35_error_message() result(msg)
        character(:), allocatable :: msg
        character(kind=c_char), pointer :: p(:)
        type(c_ptr) :: cp
        integer :: n
        msg = "libq35 failed"
        cp = q35_last_error()
        if (.not. c_associated(cp)) return
        call c_f_pointer(cp, p, [4096])
        n = 0
        do while (n < 4096)
            if (p(n + 1) == achar(0)) exit
            n = n + 1
        end do
        msg = repeat(" ", n)
        msg = transfer(p(1:n), msg)
    end function q35_error_message

end module q35_status
